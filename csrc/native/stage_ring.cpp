// Native SWRING01 frame codec: 76-byte little-endian header
// <8sHHIIQQihh32s> | metadata | payload, SHA-256 (OpenSSL) over metadata||payload.
// Shares golden vectors with the Python codec (protocol/stage_ring.py); used by
// native peers and for fast validation of large frames without Python copies.
#include <openssl/evp.h>
#include <openssl/crypto.h>
#include <torch/extension.h>

#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>

namespace {

constexpr char kMagic[8] = {'S', 'W', 'R', 'I', 'N', 'G', '0', '1'};
constexpr size_t kHeader = 76;
constexpr uint64_t kMaxMeta = 4ull << 20;
constexpr uint64_t kMaxPayload = 1ull << 30;

void sha256(const uint8_t* a, size_t na, const uint8_t* b, size_t nb, uint8_t out[32]) {
  EVP_MD_CTX* ctx = EVP_MD_CTX_new();
  if (!ctx) throw std::runtime_error("EVP_MD_CTX_new failed");
  unsigned int len = 0;
  const bool ok = EVP_DigestInit_ex(ctx, EVP_sha256(), nullptr) == 1 &&
                  EVP_DigestUpdate(ctx, a, na) == 1 && EVP_DigestUpdate(ctx, b, nb) == 1 &&
                  EVP_DigestFinal_ex(ctx, out, &len) == 1;
  EVP_MD_CTX_free(ctx);
  if (!ok || len != 32) throw std::runtime_error("SHA-256 failed");
}

template <typename T>
void put(std::string& s, size_t off, T v) {
  std::memcpy(&s[off], &v, sizeof(T));  // little-endian host (x86-64 / aarch64)
}

template <typename T>
T get(const std::string& s, size_t off) {
  T v;
  std::memcpy(&v, s.data() + off, sizeof(T));
  return v;
}

}  // namespace

pybind11::bytes ring_encode(int64_t op, int64_t flags, int64_t seq, int64_t pos, int64_t src,
                            int64_t dst, const std::string& meta, const std::string& payload) {
  if (meta.size() > kMaxMeta) throw std::invalid_argument("metadata exceeds 4 MiB");
  if (payload.size() > kMaxPayload) throw std::invalid_argument("payload exceeds 1 GiB");
  if (src < -1 || src > 32767 || dst < -1 || dst > 32767) throw std::invalid_argument("stage id");
  if (op < 1 || op > 13) throw std::invalid_argument("unknown operation");
  std::string f(kHeader + meta.size() + payload.size(), '\0');
  std::memcpy(&f[0], kMagic, 8);
  put<uint16_t>(f, 8, 1);
  put<uint16_t>(f, 10, static_cast<uint16_t>(op));
  put<uint32_t>(f, 12, static_cast<uint32_t>(flags));
  put<uint32_t>(f, 16, static_cast<uint32_t>(meta.size()));
  put<uint64_t>(f, 20, static_cast<uint64_t>(payload.size()));
  put<uint64_t>(f, 28, static_cast<uint64_t>(seq));
  put<int32_t>(f, 36, static_cast<int32_t>(pos));
  put<int16_t>(f, 40, static_cast<int16_t>(src));
  put<int16_t>(f, 42, static_cast<int16_t>(dst));
  uint8_t digest[32];
  sha256(reinterpret_cast<const uint8_t*>(meta.data()), meta.size(),
         reinterpret_cast<const uint8_t*>(payload.data()), payload.size(), digest);
  std::memcpy(&f[44], digest, 32);
  std::memcpy(&f[kHeader], meta.data(), meta.size());
  std::memcpy(&f[kHeader + meta.size()], payload.data(), payload.size());
  return pybind11::bytes(f);
}

// Returns (op, flags, seq, pos, src, dst, metadata bytes, payload bytes); raises on any
// violation of magic, version, limits, lengths or checksum.
pybind11::tuple ring_decode(const std::string& f) {
  if (f.size() < kHeader) throw std::invalid_argument("short header");
  if (std::memcmp(f.data(), kMagic, 8) != 0) throw std::invalid_argument("bad magic");
  if (get<uint16_t>(f, 8) != 1) throw std::invalid_argument("unsupported version");
  const uint16_t op = get<uint16_t>(f, 10);
  if (op < 1 || op > 13) throw std::invalid_argument("unknown operation");
  const uint32_t mlen = get<uint32_t>(f, 16);
  const uint64_t plen = get<uint64_t>(f, 20);
  if (mlen > kMaxMeta || plen > kMaxPayload) throw std::invalid_argument("component too large");
  if (f.size() != kHeader + mlen + plen) throw std::invalid_argument("length mismatch");
  const int16_t src = get<int16_t>(f, 40), dst = get<int16_t>(f, 42);
  if (src < -1 || dst < -1) throw std::invalid_argument("stage id");
  const int32_t pos = get<int32_t>(f, 36);
  if (pos < -1) throw std::invalid_argument("token position");
  uint8_t digest[32];
  sha256(reinterpret_cast<const uint8_t*>(f.data() + kHeader), mlen,
         reinterpret_cast<const uint8_t*>(f.data() + kHeader + mlen), plen, digest);
  if (CRYPTO_memcmp(digest, f.data() + 44, 32) != 0) throw std::invalid_argument("checksum mismatch");
  return pybind11::make_tuple(static_cast<int64_t>(op), static_cast<int64_t>(get<uint32_t>(f, 12)),
                              static_cast<int64_t>(get<uint64_t>(f, 28)), static_cast<int64_t>(pos),
                              static_cast<int64_t>(src), static_cast<int64_t>(dst),
                              pybind11::bytes(f.substr(kHeader, mlen)),
                              pybind11::bytes(f.substr(kHeader + mlen, plen)));
}
