// CPU oracle for one SwiGLU expert: y = W_down (silu(W_gate x) * (W_up x)).
// Weight layouts: gate/up [I, H] row-major, down [H, I] row-major, rows of x
// independent.  Formats (the semantics the GPU kernels are checked against):
//   f32   - fp32 weights and activations;
//   bf16  - bf16 weights (uint16 bit patterns), fp32 accumulation;
//   int4  - 4-bit weights packed two per byte (low nibble first), value
//           (q - 8) * scale, one bf16 scale per 32 consecutive inputs (g32);
//   fp8   - e4m3 weights with one fp32 scale per 128x128 weight block and
//           activations quantised to e4m3 per 1x128 block (absmax / 448),
//           the DeepSeek-V3 / Kimi-K2 block-scaled format.
// Accumulation is fp32 in a fixed order (inner index ascending), rows in parallel.
// Reference semantics: the C ABI swarm_moe_swiglu_{f32,bf16,int4_g32} of
// integrations/colibri/adapter/swarm_moe_runtime.c:39-164 and the block
// dequantisation of si/backends/colibri/sparse_moe.py:146-244.
#include <ATen/Parallel.h>
#include <torch/extension.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

namespace {

inline float bf16_to_f32(uint16_t v) {
  uint32_t u = static_cast<uint32_t>(v) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

inline float silu(float x) { return x / (1.0f + std::exp(-x)); }

// e4m3 (finite variant: no infinities, 0x7f/0xff NaN) to fp32.
inline float e4m3_to_f32(uint8_t v) {
  const int s = v >> 7, e = (v >> 3) & 0xF, m = v & 7;
  float r;
  if (e == 0) r = std::ldexp(static_cast<float>(m), -9);           // subnormal: m/8 * 2^-6
  else if (e == 15 && m == 7) r = NAN;
  else r = std::ldexp(1.0f + m / 8.0f, e - 7);
  return s ? -r : r;
}

// Round-to-nearest-even fp32 -> e4m3 with saturation to +-448.
inline uint8_t f32_to_e4m3(float x) {
  if (std::isnan(x)) return 0x7f;
  const uint8_t sign = std::signbit(x) ? 0x80 : 0;
  float a = std::fabs(x);
  if (a >= 448.0f) return sign | 0x7e;
  // Brute-force nearest over the 127 finite magnitudes (exact, used only by tests).
  uint8_t best = 0;
  float bd = INFINITY;
  for (int c = 0; c < 0x7f; ++c) {
    const float v = e4m3_to_f32(static_cast<uint8_t>(c));
    const float d = std::fabs(v - a);
    if (d < bd || (d == bd && (c & 1) == 0)) { bd = d; best = static_cast<uint8_t>(c); }
  }
  return sign | best;
}

template <typename G, typename U, typename D>
void swiglu_rows(const float* x, int64_t rows, int64_t H, int64_t I, G gate, U up, D down,
                 float* y) {
  at::parallel_for(0, rows, 1, [&](int64_t r0, int64_t r1) {
  for (int64_t r = r0; r < r1; ++r) {
    const float* xr = x + r * H;
    std::vector<float> a(I);
    for (int64_t i = 0; i < I; ++i) {
      float g = 0.f, u = 0.f;
      for (int64_t h = 0; h < H; ++h) {
        g += gate(i, h) * xr[h];
        u += up(i, h) * xr[h];
      }
      a[i] = silu(g) * u;
    }
    for (int64_t h = 0; h < H; ++h) {
      float acc = 0.f;
      for (int64_t i = 0; i < I; ++i) acc += down(h, i) * a[i];
      y[r * H + h] = acc;
    }
  }
  });
}

}  // namespace

at::Tensor swiglu_f32(const at::Tensor& x, const at::Tensor& g, const at::Tensor& u,
                      const at::Tensor& d) {
  auto xc = x.contiguous().to(at::kFloat), gc = g.contiguous().to(at::kFloat),
       uc = u.contiguous().to(at::kFloat), dc = d.contiguous().to(at::kFloat);
  const int64_t R = xc.size(0), H = xc.size(1), I = gc.size(0);
  auto y = at::empty({R, H}, xc.options());
  const float *G = gc.data_ptr<float>(), *U = uc.data_ptr<float>(), *D = dc.data_ptr<float>();
  swiglu_rows(xc.data_ptr<float>(), R, H, I, [&](int64_t i, int64_t h) { return G[i * H + h]; },
              [&](int64_t i, int64_t h) { return U[i * H + h]; },
              [&](int64_t h, int64_t i) { return D[h * I + i]; }, y.data_ptr<float>());
  return y;
}

at::Tensor swiglu_bf16(const at::Tensor& x, const at::Tensor& g, const at::Tensor& u,
                       const at::Tensor& d) {
  TORCH_CHECK(g.scalar_type() == at::kBFloat16, "bf16 weights");
  auto xc = x.contiguous().to(at::kFloat);
  auto gc = g.contiguous(), uc = u.contiguous(), dc = d.contiguous();
  const int64_t R = xc.size(0), H = xc.size(1), I = gc.size(0);
  auto y = at::empty({R, H}, xc.options());
  const uint16_t* G = reinterpret_cast<const uint16_t*>(gc.data_ptr());
  const uint16_t* U = reinterpret_cast<const uint16_t*>(uc.data_ptr());
  const uint16_t* D = reinterpret_cast<const uint16_t*>(dc.data_ptr());
  swiglu_rows(xc.data_ptr<float>(), R, H, I,
              [&](int64_t i, int64_t h) { return bf16_to_f32(G[i * H + h]); },
              [&](int64_t i, int64_t h) { return bf16_to_f32(U[i * H + h]); },
              [&](int64_t h, int64_t i) { return bf16_to_f32(D[h * I + i]); },
              y.data_ptr<float>());
  return y;
}

// Packed int4 g32: q[rows, cols/2] uint8, scales[rows, cols/32] bf16.
static inline float int4_at(const uint8_t* q, const uint16_t* s, int64_t cols, int64_t r,
                            int64_t c) {
  const uint8_t b = q[r * (cols / 2) + c / 2];
  const int v = (c & 1) ? (b >> 4) : (b & 0xF);
  return static_cast<float>(v - 8) * bf16_to_f32(s[r * (cols / 32) + c / 32]);
}

at::Tensor swiglu_int4_g32(const at::Tensor& x, const at::Tensor& gq, const at::Tensor& gs,
                           const at::Tensor& uq, const at::Tensor& us, const at::Tensor& dq,
                           const at::Tensor& ds) {
  auto xc = x.contiguous().to(at::kFloat);
  const int64_t R = xc.size(0), H = xc.size(1), I = gq.size(0);
  TORCH_CHECK(H % 32 == 0 && I % 32 == 0, "int4 g32 needs dims % 32");
  auto y = at::empty({R, H}, xc.options());
  auto G = gq.contiguous(), GS = gs.contiguous(), Uq = uq.contiguous(), US = us.contiguous(),
       Dq = dq.contiguous(), DS = ds.contiguous();
  const uint8_t *g = G.data_ptr<uint8_t>(), *u = Uq.data_ptr<uint8_t>(), *dd = Dq.data_ptr<uint8_t>();
  const uint16_t* gsc = reinterpret_cast<const uint16_t*>(GS.data_ptr());
  const uint16_t* usc = reinterpret_cast<const uint16_t*>(US.data_ptr());
  const uint16_t* dsc = reinterpret_cast<const uint16_t*>(DS.data_ptr());
  swiglu_rows(xc.data_ptr<float>(), R, H, I,
              [&](int64_t i, int64_t h) { return int4_at(g, gsc, H, i, h); },
              [&](int64_t i, int64_t h) { return int4_at(u, usc, H, i, h); },
              [&](int64_t h, int64_t i) { return int4_at(dd, dsc, I, h, i); }, y.data_ptr<float>());
  return y;
}

// fp8 block-scaled GEMM oracle: y[R, N] = dequant(xq, xs) . dequant(wq, ws)^T, where
// xq [R, K] e4m3 with xs [R, K/128] fp32, wq [N, K] e4m3 with ws [N/128, K/128] fp32.
at::Tensor fp8_block_gemm(const at::Tensor& xq, const at::Tensor& xs, const at::Tensor& wq,
                          const at::Tensor& ws) {
  const int64_t R = xq.size(0), K = xq.size(1), N = wq.size(0);
  TORCH_CHECK(K % 128 == 0, "K % 128");
  auto X = xq.contiguous(), XS = xs.contiguous().to(at::kFloat), W = wq.contiguous(),
       WS = ws.contiguous().to(at::kFloat);
  const uint8_t* x = reinterpret_cast<const uint8_t*>(X.data_ptr());
  const uint8_t* w = reinterpret_cast<const uint8_t*>(W.data_ptr());
  const float* xsp = XS.data_ptr<float>();
  const float* wsp = WS.data_ptr<float>();
  auto y = at::empty({R, N}, at::TensorOptions().dtype(at::kFloat));
  float* yp = y.data_ptr<float>();
  const int64_t KB = K / 128;
  at::parallel_for(0, R, 1, [&](int64_t r0, int64_t r1) {
  for (int64_t r = r0; r < r1; ++r)
    for (int64_t n = 0; n < N; ++n) {
      float acc = 0.f;
      for (int64_t kb = 0; kb < KB; ++kb) {
        float part = 0.f;
        for (int64_t k = kb * 128; k < kb * 128 + 128; ++k)
          part += e4m3_to_f32(x[r * K + k]) * e4m3_to_f32(w[n * K + k]);
        acc += part * xsp[r * KB + kb] * wsp[(n / 128) * KB + kb];
      }
      yp[r * N + n] = acc;
    }
  });
  return y;
}

// Quantise fp32 rows to e4m3 with one scale per 1x128 block (scale = absmax / 448).
std::vector<at::Tensor> quant_fp8_1x128(const at::Tensor& x) {
  auto X = x.contiguous().to(at::kFloat);
  const int64_t R = X.size(0), K = X.size(1);
  TORCH_CHECK(K % 128 == 0, "K % 128");
  auto q = at::empty({R, K}, at::TensorOptions().dtype(at::kByte));
  auto s = at::empty({R, K / 128}, at::TensorOptions().dtype(at::kFloat));
  const float* xp = X.data_ptr<float>();
  uint8_t* qp = q.data_ptr<uint8_t>();
  float* sp = s.data_ptr<float>();
  for (int64_t r = 0; r < R; ++r)
    for (int64_t b = 0; b < K / 128; ++b) {
      float amax = 0.f;
      for (int64_t k = b * 128; k < b * 128 + 128; ++k) amax = std::max(amax, std::fabs(xp[r * K + k]));
      const float sc = amax > 0.f ? amax / 448.0f : 1.0f;
      sp[r * (K / 128) + b] = sc;
      for (int64_t k = b * 128; k < b * 128 + 128; ++k) qp[r * K + k] = f32_to_e4m3(xp[r * K + k] / sc);
    }
  return {q, s};
}

at::Tensor e4m3_decode(const at::Tensor& q) {
  auto Q = q.contiguous();
  auto out = at::empty(Q.sizes(), at::TensorOptions().dtype(at::kFloat));
  const uint8_t* qp = reinterpret_cast<const uint8_t*>(Q.data_ptr());
  float* op = out.data_ptr<float>();
  for (int64_t i = 0; i < Q.numel(); ++i) op[i] = e4m3_to_f32(qp[i]);
  return out;
}
