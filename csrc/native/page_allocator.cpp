// Host-side paged-KV page allocator: LIFO free list with per-page reference
// counts (copy-on-write prefix sharing), O(1) alloc/release per page.  The
// Python PagedKVCache uses it when the native library is built.
#include <torch/extension.h>

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

class NativePageAllocator {
 public:
  explicit NativePageAllocator(int64_t n) : ref_(n, 0) {
    free_.reserve(n);
    for (int64_t p = n - 1; p >= 0; --p) free_.push_back(static_cast<int32_t>(p));
  }
  int64_t num_pages() const { return static_cast<int64_t>(ref_.size()); }
  int64_t free() const { return static_cast<int64_t>(free_.size()); }
  std::vector<int32_t> alloc(int64_t n) {
    if (n < 0 || static_cast<size_t>(n) > free_.size())
      throw std::runtime_error("out of KV pages: need " + std::to_string(n) + ", free " +
                               std::to_string(free_.size()));
    std::vector<int32_t> out(n);
    for (int64_t i = 0; i < n; ++i) {
      out[i] = free_.back();
      free_.pop_back();
      ref_[out[i]] = 1;
    }
    return out;
  }
  void retain(const std::vector<int32_t>& pages) {
    for (int32_t p : pages) {
      check(p);
      if (ref_[p] <= 0) throw std::runtime_error("retain of a free page");
      ++ref_[p];
    }
  }
  void release(const std::vector<int32_t>& pages) {
    for (int32_t p : pages) {
      check(p);
      if (ref_[p] <= 0) throw std::runtime_error("page " + std::to_string(p) + " released twice");
      if (--ref_[p] == 0) free_.push_back(p);
    }
  }
  int64_t refcount(int32_t p) const {
    check(p);
    return ref_[p];
  }

 private:
  void check(int32_t p) const {
    if (p < 0 || static_cast<size_t>(p) >= ref_.size()) throw std::out_of_range("page id");
  }
  std::vector<int32_t> free_;
  std::vector<int32_t> ref_;
};

void bind_page_allocator(pybind11::module& m) {
  pybind11::class_<NativePageAllocator>(m, "PageAllocator")
      .def(pybind11::init<int64_t>())
      .def_property_readonly("num_pages", &NativePageAllocator::num_pages)
      .def_property_readonly("free", &NativePageAllocator::free)
      .def("alloc", &NativePageAllocator::alloc)
      .def("retain", &NativePageAllocator::retain)
      .def("release", &NativePageAllocator::release)
      .def("refcount", &NativePageAllocator::refcount);
}
