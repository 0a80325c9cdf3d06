// AdamW over a list of f32 parameters in one launch: the aux-Adam groups of
// SingleDeviceMuonMDWithAuxAdam (optimizer/muon.py:616-650 with adam_update
// at :131-136): exp_avg.lerp_(g, 1-b1); exp_avg_sq.lerp_(g*g, 1-b2);
// update = (exp_avg / (1 - b1^t)) / (sqrt(exp_avg_sq / (1 - b2^t)) + eps);
// p *= 1 - lr*wd; p -= lr * update.  The reference's eleven tensor passes per
// parameter become one read of (p, g, m1, m2) and one write of (p, m1, m2),
// optionally with a bf16 copy of the new p for the next forward's GEMMs.
//
// The arithmetic follows the torch formulation operation by operation (f32,
// each product, quotient and square root rounded on its own):
//   step on the device (capturable): the bias corrections 1 - b^t are f32
//     device scalars and the moments are divided by them; with a host step
//     the moments are multiplied by the f32 reciprocal of the host's
//     (double) correction, as torch does for a Python-scalar divisor;
//   lr on the device: decay = 1 - lr*wd in f32 and p = p*decay - lr*update;
//     with a host lr: decay is the host's value and p = fma(-lr, update,
//     p*decay) (torch's add_ with alpha = -lr).
#include "zs_common.cuh"

namespace zs {
namespace adam {

constexpr int MAXT = 96;           // tensors per launch
constexpr int THREADS = 256;
constexpr int CHUNK = THREADS * 8; // elements per block iteration: two groups of four per thread

struct List {
  int count;
  int64_t chunk_start[MAXT + 1];   // prefix of chunks per tensor
  zs_adamw_tensor t[MAXT];
};

struct Hyper {
  const float* lr_dev;  // nullable
  float lr_host;
  float decay_host;     // 1 - lr*wd from the host (used with lr_host)
  float w1, w2;         // 1 - b1, 1 - b2 (rounded from double on the host)
  float b1, b2;         // the betas as f32, for b^t with a device step
  float eps, wd;
};

__device__ __forceinline__ float lerp_t(float a, float b, float w) {
  const float d = b - a;
  return w < 0.5f ? a + w * d : b - d * (1.f - w);
}

struct Coef {
  bool div;             // bias corrections are divisors (device step) or reciprocals (host step)
  bool dev_lr;
  float bc1, bc2, lr, decay;
};

__device__ __forceinline__ void adam_elem(float& p, float g, float& m1, float& m2, const Hyper& h, const Coef& c) {
  m1 = lerp_t(m1, g, h.w1);
  m2 = lerp_t(m2, __fmul_rn(g, g), h.w2);
  const float c1 = c.div ? __fdiv_rn(m1, c.bc1) : __fmul_rn(m1, c.bc1);
  const float c2 = c.div ? __fdiv_rn(m2, c.bc2) : __fmul_rn(m2, c.bc2);
  const float u = __fdiv_rn(c1, __fadd_rn(__fsqrt_rn(c2), h.eps));
  const float pd = __fmul_rn(p, c.decay);
  p = c.dev_lr ? __fsub_rn(pd, __fmul_rn(c.lr, u)) : __fmaf_rn(-c.lr, u, pd);
}

__global__ void __launch_bounds__(THREADS) adamw_kernel(List L, Hyper h) {
  const int64_t total = L.chunk_start[L.count];
  Coef c;
  c.dev_lr = h.lr_dev != nullptr;
  c.lr = c.dev_lr ? __ldg(h.lr_dev) : h.lr_host;
  c.decay = c.dev_lr ? __fsub_rn(1.f, __fmul_rn(c.lr, h.wd)) : h.decay_host;
  for (int64_t ch = blockIdx.x; ch < total; ch += gridDim.x) {
    int lo = 0, hi = L.count - 1;   // the tensor owning chunk ch: last i with chunk_start[i] <= ch
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (L.chunk_start[mid] <= ch) lo = mid; else hi = mid - 1;
    }
    const zs_adamw_tensor& T = L.t[lo];
    c.div = T.step_dev != nullptr;
    if (c.div) {
      const float t = __ldg(T.step_dev);
      c.bc1 = __fsub_rn(1.f, powf(h.b1, t));
      c.bc2 = __fsub_rn(1.f, powf(h.b2, t));
    } else {
      c.bc1 = T.inv_bc1_host;
      c.bc2 = T.inv_bc2_host;
    }
    const int64_t n = T.n;
    __nv_bfloat16* sh = reinterpret_cast<__nv_bfloat16*>(T.shadow_bf16);
    const bool vec = ((reinterpret_cast<uintptr_t>(T.p) | reinterpret_cast<uintptr_t>(T.g) |
                       reinterpret_cast<uintptr_t>(T.m1) | reinterpret_cast<uintptr_t>(T.m2)) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(sh) & 7) == 0;
    const int64_t base = (ch - L.chunk_start[lo]) * CHUNK + (int64_t)threadIdx.x * 4;
#pragma unroll
    for (int gi = 0; gi < 2; ++gi) {
      const int64_t e = base + (int64_t)gi * THREADS * 4;
      if (vec && e + 4 <= n) {
        const float4 p4 = *reinterpret_cast<const float4*>(T.p + e);
        const float4 g4 = __ldg(reinterpret_cast<const float4*>(T.g + e));
        const float4 a4 = *reinterpret_cast<const float4*>(T.m1 + e);
        const float4 b4 = *reinterpret_cast<const float4*>(T.m2 + e);
        float pv[4] = {p4.x, p4.y, p4.z, p4.w}, av[4] = {a4.x, a4.y, a4.z, a4.w};
        float bv[4] = {b4.x, b4.y, b4.z, b4.w};
        const float gv[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) adam_elem(pv[k], gv[k], av[k], bv[k], h, c);
        *reinterpret_cast<float4*>(T.p + e) = make_float4(pv[0], pv[1], pv[2], pv[3]);
        *reinterpret_cast<float4*>(T.m1 + e) = make_float4(av[0], av[1], av[2], av[3]);
        *reinterpret_cast<float4*>(T.m2 + e) = make_float4(bv[0], bv[1], bv[2], bv[3]);
        if (sh != nullptr) {
          __nv_bfloat162 lo2 = __floats2bfloat162_rn(pv[0], pv[1]), hi2 = __floats2bfloat162_rn(pv[2], pv[3]);
          uint2 w;
          w.x = *reinterpret_cast<uint32_t*>(&lo2);
          w.y = *reinterpret_cast<uint32_t*>(&hi2);
          *reinterpret_cast<uint2*>(sh + e) = w;
        }
      } else {
        for (int k = 0; k < 4 && e + k < n; ++k) {
          const int64_t i = e + k;
          float pv = T.p[i], av = T.m1[i], bv = T.m2[i];
          adam_elem(pv, T.g[i], av, bv, h, c);
          T.p[i] = pv;
          T.m1[i] = av;
          T.m2[i] = bv;
          if (sh != nullptr) sh[i] = __float2bfloat16_rn(pv);
        }
      }
    }
  }
}

}  // namespace adam
}  // namespace zs

extern "C" int zs_adamw_step(const zs_adamw_tensor* tensors, int count, const float* lr_dev, float lr_host,
                             float decay_host, float b1, float b2, double one_minus_b1, double one_minus_b2,
                             float eps, float weight_decay, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ZS_REQUIRE(count >= 0 && (count == 0 || tensors != nullptr), ZS_ERR_ARG);
  const void* first = nullptr;
  for (int i = 0; i < count; ++i) {
    const zs_adamw_tensor& t = tensors[i];
    ZS_REQUIRE(t.n >= 0, ZS_ERR_SHAPE);
    ZS_REQUIRE(t.n == 0 || (t.p && t.g && t.m1 && t.m2), ZS_ERR_ARG);
    if (first == nullptr && t.n > 0) first = t.p;
  }
  if (first == nullptr) return ZS_OK;
  ZS_BIND(first);
  const zs::adam::Hyper h{lr_dev, lr_host, decay_host, (float)one_minus_b1, (float)one_minus_b2, b1, b2, eps,
                          weight_decay};
  int i = 0;
  while (i < count) {
    zs::adam::List L{};
    L.count = 0;
    L.chunk_start[0] = 0;
    for (; i < count && L.count < zs::adam::MAXT; ++i) {
      if (tensors[i].n == 0) continue;
      L.t[L.count] = tensors[i];
      L.chunk_start[L.count + 1] = L.chunk_start[L.count] + (tensors[i].n + zs::adam::CHUNK - 1) / zs::adam::CHUNK;
      ++L.count;
    }
    if (L.count == 0) continue;
    int64_t blocks = L.chunk_start[L.count];
    if (blocks > 148 * 8) blocks = 148 * 8;
    zs::adam::adamw_kernel<<<(unsigned)blocks, zs::adam::THREADS, 0, stream>>>(L, h);
    ZS_CUDA_TRY(cudaGetLastError());
  }
  return ZS_OK;
}
