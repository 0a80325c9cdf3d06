// Bandwidth-bound kernels around attention:
//   * zero-centred RMSNorm forward/backward (modeling/zRMSNorm.py:4-20):
//       y = x * rsqrt(mean(x^2) + eps) * (1 + w), computed in f32, stored in
//       the input dtype; backward gives dx and the f32 weight gradient.
//   * rotate-half RoPE with separate Q/K cos/sin tables, in place
//     (modeling/liger_rope.py:20-119): pairs (i, i + hd/2) of every head are
//     rotated by the row's angle; the backward rotates by the negative angle.
#include "zs_common.cuh"

namespace zs {

template <typename T>
__device__ __forceinline__ float ldf(const T* p) {
  return to_f32<T>(*p);
}

// One warp per row; each lane keeps its slice of the row in registers when
// d <= 32 * MAXV (else the row is re-read from L1/L2).
template <typename T, typename W>
__global__ void zrmsnorm_fwd_kernel(const T* __restrict__ x, const W* __restrict__ w, T* __restrict__ y,
                                    float* __restrict__ rstd, int64_t rows, int d, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const T* xr = x + r * d;
    float ss = 0.f;
    for (int c = lane; c < d; c += 32) {
      const float v = ldf(xr + c);
      ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    // torch: x.pow(2).mean(-1) + eps, then rsqrt, all f32
    const float rs = rsqrtf(ss / (float)d + eps);
    if (lane == 0 && rstd != nullptr) rstd[r] = rs;
    T* yr = y + r * d;
    for (int c = lane; c < d; c += 32) yr[c] = from_f32<T>((ldf(xr + c) * rs) * (1.0f + ldf(w + c)));
  }
}

// dx = rs * (dn - n * mean(dn * n)),  dn = dy * (1 + w),  n = x * rs;
// dw partial sums per block: part[blockIdx][c] = sum over this block's rows of dy * n.
template <typename T, typename W>
__global__ void zrmsnorm_bwd_kernel(const T* __restrict__ dy, const T* __restrict__ x, const W* __restrict__ w,
                                    const float* __restrict__ rstd, T* __restrict__ dx, float* __restrict__ dw_part,
                                    int64_t rows, int d) {
  extern __shared__ float sdw[];  // [d] per block
  for (int c = threadIdx.x; c < d; c += blockDim.x) sdw[c] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const T* xr = x + r * d;
    const T* dyr = dy + r * d;
    const float rs = rstd[r];
    float dot = 0.f;
    for (int c = lane; c < d; c += 32) {
      const float n = ldf(xr + c) * rs;
      const float g = ldf(dyr + c);
      dot = fmaf(g * (1.0f + ldf(w + c)), n, dot);
      atomicAdd(&sdw[c], g * n);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
    const float mean = dot / (float)d;
    T* dxr = dx + r * d;
    for (int c = lane; c < d; c += 32) {
      const float n = ldf(xr + c) * rs;
      const float dn = ldf(dyr + c) * (1.0f + ldf(w + c));
      dxr[c] = from_f32<T>(rs * (dn - n * mean));
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < d; c += blockDim.x) dw_part[(int64_t)blockIdx.x * d + c] = sdw[c];
}

// Vectorised backward for rows of d = 128 * NV elements: lane holds NV chunks
// of 4 consecutive columns (x, dy and the dw accumulators in registers); the
// block's 8 warps reduce their dw through shared memory without atomics.
template <typename T>
struct Vec4;
template <>
struct Vec4<float> {
  using type = float4;
  __device__ static void unpack(const float4& v, float (&o)[4]) { o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w; }
  __device__ static float4 pack(const float (&o)[4]) { return make_float4(o[0], o[1], o[2], o[3]); }
};
template <>
struct Vec4<__nv_bfloat16> {
  using type = uint2;
  __device__ static void unpack(const uint2& v, float (&o)[4]) {
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.y));
    o[0] = a.x; o[1] = a.y; o[2] = b.x; o[3] = b.y;
  }
  __device__ static uint2 pack(const float (&o)[4]) {
    __nv_bfloat162 a = __floats2bfloat162_rn(o[0], o[1]), b = __floats2bfloat162_rn(o[2], o[3]);
    return make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
  }
};
template <>
struct Vec4<__half> {
  using type = uint2;
  __device__ static void unpack(const uint2& v, float (&o)[4]) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
    o[0] = a.x; o[1] = a.y; o[2] = b.x; o[3] = b.y;
  }
  __device__ static uint2 pack(const float (&o)[4]) {
    __half2 a = __floats2half2_rn(o[0], o[1]), b = __floats2half2_rn(o[2], o[3]);
    return make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
  }
};

template <typename T, typename W, int NV>
__global__ void __launch_bounds__(256) zrmsnorm_bwd_vec_kernel(const T* __restrict__ dy, const T* __restrict__ x,
                                                               const W* __restrict__ w, const float* __restrict__ rstd,
                                                               T* __restrict__ dx, float* __restrict__ dw_part,
                                                               int64_t rows) {
  constexpr int D = 128 * NV;
  using V = Vec4<T>;
  using VT = typename V::type;
  extern __shared__ float sdw[];  // [8][D] per-warp dw, then [D] of (1 + w)
  float* swp = sdw + 8 * D;
  for (int c = threadIdx.x; c < D; c += blockDim.x) swp[c] = 1.0f + to_f32<W>(w[c]);
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float acc[NV][4];
#pragma unroll
  for (int j = 0; j < NV; ++j)
#pragma unroll
    for (int v = 0; v < 4; ++v) acc[j][v] = 0.f;
  const int64_t warps = (int64_t)gridDim.x * 8;
  for (int64_t r = (int64_t)blockIdx.x * 8 + warp; r < rows; r += warps) {
    const VT* xr = reinterpret_cast<const VT*>(x + r * D);
    const VT* gr = reinterpret_cast<const VT*>(dy + r * D);
    const float rs = __ldg(rstd + r);
    float xv[NV][4], gv[NV][4];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      V::unpack(xr[j * 32 + lane], xv[j]);
      V::unpack(gr[j * 32 + lane], gv[j]);
    }
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j)
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const int c = (j * 32 + lane) * 4 + v;
        const float n = xv[j][v] * rs;
        dot = fmaf(gv[j][v] * swp[c], n, dot);
        acc[j][v] = fmaf(gv[j][v], n, acc[j][v]);
      }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
    const float mean = dot / (float)D;
    VT* dxr = reinterpret_cast<VT*>(dx + r * D);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      float o[4];
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const int c = (j * 32 + lane) * 4 + v;
        const float n = xv[j][v] * rs;
        o[v] = rs * (gv[j][v] * swp[c] - n * mean);
      }
      dxr[j * 32 + lane] = V::pack(o);
    }
  }
#pragma unroll
  for (int j = 0; j < NV; ++j)
#pragma unroll
    for (int v = 0; v < 4; ++v) sdw[warp * D + (j * 32 + lane) * 4 + v] = acc[j][v];
  __syncthreads();
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float t = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) t += sdw[q * D + c];
    dw_part[(int64_t)blockIdx.x * D + c] = t;
  }
}

// Residual add fused with the norm, for an f32 residual stream x and a bf16
// branch r (the transformer block's `x + branch` followed by a norm whose output
// feeds bf16 GEMMs):  h = x + r (f32, stored when h_out is given), y = bf16 of
// zRMSNorm(h).  Without r it is the norm of x with a bf16 output.  Rows of
// d = 128 * NV f32 values; warp per row, lane holds NV chunks of 4 columns.
template <int NV>
__global__ void __launch_bounds__(256) add_zrmsnorm_fwd_kernel(const float* __restrict__ x,
                                                               const __nv_bfloat16* __restrict__ r,
                                                               const float* __restrict__ w,
                                                               float* __restrict__ h_out,
                                                               __nv_bfloat16* __restrict__ y,
                                                               float* __restrict__ rstd, int64_t rows, float eps) {
  constexpr int D = 128 * NV;
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows; row += warps) {
    const float4* xr = reinterpret_cast<const float4*>(x + row * D);
    float hv[NV][4];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const float4 a = __ldg(xr + j * 32 + lane);
      hv[j][0] = a.x; hv[j][1] = a.y; hv[j][2] = a.z; hv[j][3] = a.w;
    }
    if (r != nullptr) {
      const uint2* rr = reinterpret_cast<const uint2*>(r + row * D);
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        float b[4];
        Vec4<__nv_bfloat16>::unpack(__ldg(rr + j * 32 + lane), b);
#pragma unroll
        for (int v = 0; v < 4; ++v) hv[j][v] = hv[j][v] + b[v];
      }
      if (h_out != nullptr) {
        float4* hr = reinterpret_cast<float4*>(h_out + row * D);
#pragma unroll
        for (int j = 0; j < NV; ++j) hr[j * 32 + lane] = make_float4(hv[j][0], hv[j][1], hv[j][2], hv[j][3]);
      }
    }
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j)
#pragma unroll
      for (int v = 0; v < 4; ++v) ss = fmaf(hv[j][v], hv[j][v], ss);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float rs = rsqrtf(ss / (float)D + eps);
    if (lane == 0 && rstd != nullptr) rstd[row] = rs;
    const float4* wr = reinterpret_cast<const float4*>(w);
    uint2* yr = reinterpret_cast<uint2*>(y + row * D);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const float4 wv = __ldg(wr + j * 32 + lane);
      const float o[4] = {(hv[j][0] * rs) * (1.0f + wv.x), (hv[j][1] * rs) * (1.0f + wv.y),
                          (hv[j][2] * rs) * (1.0f + wv.z), (hv[j][3] * rs) * (1.0f + wv.w)};
      yr[j * 32 + lane] = Vec4<__nv_bfloat16>::pack(o);
    }
  }
}

// Backward of add_zrmsnorm_fwd_kernel: dy bf16, h (the saved f32 norm input),
// dh_in (optional f32: the gradient reaching h from its other use, the residual
// path); dx = dh_in + the norm's input gradient (f32, the gradient of x), dr =
// bf16 of dx (optional, the gradient of the bf16 branch r); dweight partials per
// block as zrmsnorm_bwd_vec_kernel.
template <int NV>
__global__ void __launch_bounds__(256) add_zrmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy,
                                                               const float* __restrict__ h,
                                                               const float* __restrict__ w,
                                                               const float* __restrict__ rstd,
                                                               const float* __restrict__ dh_in,
                                                               float* __restrict__ dx,
                                                               __nv_bfloat16* __restrict__ dr,
                                                               float* __restrict__ dw_part, int64_t rows) {
  constexpr int D = 128 * NV;
  extern __shared__ float sdw[];  // [8][D] per-warp dw, then [D] of (1 + w)
  float* swp = sdw + 8 * D;
  for (int c = threadIdx.x; c < D; c += blockDim.x) swp[c] = 1.0f + w[c];
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float acc[NV][4];
#pragma unroll
  for (int j = 0; j < NV; ++j)
#pragma unroll
    for (int v = 0; v < 4; ++v) acc[j][v] = 0.f;
  const int64_t warps = (int64_t)gridDim.x * 8;
  for (int64_t row = (int64_t)blockIdx.x * 8 + warp; row < rows; row += warps) {
    const float4* hr = reinterpret_cast<const float4*>(h + row * D);
    const uint2* gr = reinterpret_cast<const uint2*>(dy + row * D);
    const float rs = __ldg(rstd + row);
    float xv[NV][4], gv[NV][4];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const float4 a = __ldg(hr + j * 32 + lane);
      xv[j][0] = a.x; xv[j][1] = a.y; xv[j][2] = a.z; xv[j][3] = a.w;
      Vec4<__nv_bfloat16>::unpack(__ldg(gr + j * 32 + lane), gv[j]);
    }
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j)
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const int c = (j * 32 + lane) * 4 + v;
        const float n = xv[j][v] * rs;
        dot = fmaf(gv[j][v] * swp[c], n, dot);
        acc[j][v] = fmaf(gv[j][v], n, acc[j][v]);
      }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
    const float mean = dot / (float)D;
    const float4* ehr = dh_in != nullptr ? reinterpret_cast<const float4*>(dh_in + row * D) : nullptr;
    float4* dxr = reinterpret_cast<float4*>(dx + row * D);
    uint2* drr = dr != nullptr ? reinterpret_cast<uint2*>(dr + row * D) : nullptr;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      float o[4];
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const int c = (j * 32 + lane) * 4 + v;
        const float n = xv[j][v] * rs;
        o[v] = rs * (gv[j][v] * swp[c] - n * mean);
      }
      if (ehr != nullptr) {
        const float4 e = __ldg(ehr + j * 32 + lane);
        o[0] = e.x + o[0]; o[1] = e.y + o[1]; o[2] = e.z + o[2]; o[3] = e.w + o[3];
      }
      dxr[j * 32 + lane] = make_float4(o[0], o[1], o[2], o[3]);
      if (drr != nullptr) drr[j * 32 + lane] = Vec4<__nv_bfloat16>::pack(o);
    }
  }
#pragma unroll
  for (int j = 0; j < NV; ++j)
#pragma unroll
    for (int v = 0; v < 4; ++v) sdw[warp * D + (j * 32 + lane) * 4 + v] = acc[j][v];
  __syncthreads();
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float t = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) t += sdw[q * D + c];
    dw_part[(int64_t)blockIdx.x * D + c] = t;
  }
}

__global__ void sum_rows_kernel(const float* __restrict__ part, int nparts, int d, float* __restrict__ out) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= d) return;
  float s = 0.f;
  for (int p = 0; p < nparts; ++p) s += part[(int64_t)p * d + c];
  out[c] = s;
}

// One block per (batch, position) row: all q heads then all k heads.
template <typename T, typename C>
__global__ void rope_kernel(T* __restrict__ q, int64_t q_row_stride, T* __restrict__ k, int64_t k_row_stride,
                            const C* __restrict__ q_cos, const C* __restrict__ q_sin, const C* __restrict__ k_cos,
                            const C* __restrict__ k_sin, int64_t cos_row_stride, int64_t rows, int seq_len,
                            int cos_bs, int n_qh, int n_kh, int hd, int backward, int rot) {
  // rot <= hd/2: only pairs p < rot are rotated (the others have cos 1, sin 0)
  const int half = hd / 2;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const int64_t b = r / seq_len, s = r % seq_len;
    const int64_t crow = (cos_bs == 1 ? s : b * seq_len + s) * cos_row_stride;
    const int total = (n_qh + n_kh) * rot;
    for (int i = threadIdx.x; i < total; i += blockDim.x) {
      const bool isq = i < n_qh * rot;
      const int j = isq ? i : i - n_qh * rot;
      const int h = j / rot, p = j - h * rot;
      T* base = isq ? q + r * q_row_stride + (int64_t)h * hd : k + r * k_row_stride + (int64_t)h * hd;
      const float c = to_f32<C>((isq ? q_cos : k_cos)[crow + p]);
      const float sn = to_f32<C>((isq ? q_sin : k_sin)[crow + p]);
      const float x1 = to_f32<T>(base[p]);
      const float x2 = to_f32<T>(base[p + half]);
      if (!backward) {
        base[p] = from_f32<T>(x1 * c - x2 * sn);
        base[p + half] = from_f32<T>(x2 * c + x1 * sn);
      } else {
        base[p] = from_f32<T>(x1 * c + x2 * sn);
        base[p + half] = from_f32<T>(x2 * c - x1 * sn);
      }
    }
  }
}

}  // namespace zs

using namespace zs;

#define ZS_DISPATCH_XW(xdt, wdt, ...)                                               \
  do {                                                                              \
    if (xdt == ZS_BF16 && wdt == ZS_F32) {                                          \
      using TX = __nv_bfloat16; using TW = float; __VA_ARGS__;                      \
    } else if (xdt == ZS_F32 && wdt == ZS_F32) {                                    \
      using TX = float; using TW = float; __VA_ARGS__;                              \
    } else if (xdt == ZS_F16 && wdt == ZS_F32) {                                    \
      using TX = __half; using TW = float; __VA_ARGS__;                             \
    } else if (xdt == ZS_BF16 && wdt == ZS_BF16) {                                  \
      using TX = __nv_bfloat16; using TW = __nv_bfloat16; __VA_ARGS__;              \
    } else {                                                                        \
      return ZS_ERR_DTYPE;                                                          \
    }                                                                               \
  } while (0)

extern "C" int zs_zrmsnorm_forward(const void* x, const void* weight, void* y, float* rstd, int64_t rows, int d,
                                   float eps, int x_dtype, int w_dtype, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ZS_REQUIRE(x && weight && y, ZS_ERR_ARG);
  ZS_REQUIRE(rows >= 0 && d >= 1, ZS_ERR_SHAPE);
  ZS_BIND(x);
  if (rows == 0) return ZS_OK;
  int64_t blocks = (rows + 7) / 8;
  if (blocks > 148 * 16) blocks = 148 * 16;
  ZS_DISPATCH_XW(x_dtype, w_dtype,
                 zrmsnorm_fwd_kernel<TX, TW><<<(unsigned)blocks, 256, 0, stream>>>(
                     reinterpret_cast<const TX*>(x), reinterpret_cast<const TW*>(weight), reinterpret_cast<TX*>(y),
                     rstd, rows, d, eps));
  ZS_CUDA_TRY(cudaGetLastError());
  return ZS_OK;
}

extern "C" size_t zs_zrmsnorm_backward_workspace(int64_t rows, int d) {
  return (size_t)296 * d * sizeof(float);
}

extern "C" int zs_zrmsnorm_backward(const void* dy, const void* x, const void* weight, const float* rstd, void* dx,
                                    float* dweight, int64_t rows, int d, int x_dtype, int w_dtype, void* workspace,
                                    size_t workspace_bytes, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ZS_REQUIRE(dy && x && weight && rstd && dx && dweight, ZS_ERR_ARG);
  ZS_REQUIRE(rows >= 0 && d >= 1 && d <= 12288, ZS_ERR_SHAPE);
  ZS_REQUIRE(workspace && workspace_bytes >= zs_zrmsnorm_backward_workspace(rows, d), ZS_ERR_WORKSPACE);
  ZS_BIND(x);
  int64_t blocks = (rows + 7) / 8;
  if (blocks > 296) blocks = 296;
  if (blocks < 1) blocks = 1;
  float* part = reinterpret_cast<float*>(workspace);
  const bool aligned = ((reinterpret_cast<uintptr_t>(dy) | reinterpret_cast<uintptr_t>(x) |
                         reinterpret_cast<uintptr_t>(dx)) & 15) == 0;
  const int nv = d % 128 == 0 ? d / 128 : 0;
  if (aligned && (nv == 1 || nv == 2 || nv == 3 || nv == 4 || nv == 6 || nv == 8 || nv == 12 || nv == 16)) {
    const size_t shv = (size_t)9 * d * sizeof(float);
    int rc = ZS_OK;
#define ZS_NORM_BWD_VEC(NVC)                                                                                   \
  ZS_DISPATCH_XW(x_dtype, w_dtype, {                                                                           \
    if (shv > 48 * 1024) {                                                                                     \
      ZS_CUDA_TRY(cudaFuncSetAttribute(zrmsnorm_bwd_vec_kernel<TX, TW, NVC>,                                   \
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)shv));                \
    }                                                                                                          \
    zrmsnorm_bwd_vec_kernel<TX, TW, NVC><<<(unsigned)blocks, 256, shv, stream>>>(                              \
        reinterpret_cast<const TX*>(dy), reinterpret_cast<const TX*>(x), reinterpret_cast<const TW*>(weight), \
        rstd, reinterpret_cast<TX*>(dx), part, rows);                                                          \
  })
    switch (nv) {
      case 1: ZS_NORM_BWD_VEC(1); break;
      case 2: ZS_NORM_BWD_VEC(2); break;
      case 3: ZS_NORM_BWD_VEC(3); break;
      case 4: ZS_NORM_BWD_VEC(4); break;
      case 6: ZS_NORM_BWD_VEC(6); break;
      case 8: ZS_NORM_BWD_VEC(8); break;
      case 12: ZS_NORM_BWD_VEC(12); break;
      default: ZS_NORM_BWD_VEC(16); break;
    }
#undef ZS_NORM_BWD_VEC
    if (rc != ZS_OK) return rc;
    ZS_CUDA_TRY(cudaGetLastError());
    sum_rows_kernel<<<(d + 255) / 256, 256, 0, stream>>>(part, (int)blocks, d, dweight);
    ZS_CUDA_TRY(cudaGetLastError());
    return ZS_OK;
  }
  const size_t sh = (size_t)d * sizeof(float);
  ZS_DISPATCH_XW(x_dtype, w_dtype, {
    if (sh > 48 * 1024) {
      ZS_CUDA_TRY(cudaFuncSetAttribute(zrmsnorm_bwd_kernel<TX, TW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)sh));
    }
    zrmsnorm_bwd_kernel<TX, TW><<<(unsigned)blocks, 256, sh, stream>>>(
        reinterpret_cast<const TX*>(dy), reinterpret_cast<const TX*>(x), reinterpret_cast<const TW*>(weight), rstd,
        reinterpret_cast<TX*>(dx), part, rows, d);
  });
  ZS_CUDA_TRY(cudaGetLastError());
  sum_rows_kernel<<<(d + 255) / 256, 256, 0, stream>>>(part, (int)blocks, d, dweight);
  ZS_CUDA_TRY(cudaGetLastError());
  return ZS_OK;
}

static bool addnorm_nv_ok(int d) {
  const int nv = d % 128 == 0 ? d / 128 : 0;
  return nv == 1 || nv == 2 || nv == 4 || nv == 8 || nv == 12 || nv == 16;
}

template <int NV>
static int launch_add_zrmsnorm_fwd(const float* x, const void* r, const float* weight, float* h_out, void* y,
                                   float* rstd, int64_t rows, float eps, cudaStream_t stream) {
  int64_t blocks = (rows + 7) / 8;
  if (blocks > 148 * 16) blocks = 148 * 16;
  add_zrmsnorm_fwd_kernel<NV><<<(unsigned)blocks, 256, 0, stream>>>(
      x, reinterpret_cast<const __nv_bfloat16*>(r), weight, h_out, reinterpret_cast<__nv_bfloat16*>(y), rstd, rows,
      eps);
  ZS_CUDA_TRY(cudaGetLastError());
  return ZS_OK;
}

template <int NV>
static int launch_add_zrmsnorm_bwd(const void* dy, const float* h, const float* weight, const float* rstd,
                                   const float* dh_in, float* dx, void* dr, float* part, int64_t blocks,
                                   int64_t rows, cudaStream_t stream) {
  const size_t shv = (size_t)9 * 128 * NV * sizeof(float);
  if (shv > 48 * 1024)
    ZS_CUDA_TRY(cudaFuncSetAttribute(add_zrmsnorm_bwd_kernel<NV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)shv));
  add_zrmsnorm_bwd_kernel<NV><<<(unsigned)blocks, 256, shv, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(dy), h, weight, rstd, dh_in, dx, reinterpret_cast<__nv_bfloat16*>(dr),
      part, rows);
  ZS_CUDA_TRY(cudaGetLastError());
  return ZS_OK;
}

extern "C" int zs_add_zrmsnorm_forward(const float* x, const void* r, const float* weight, float* h_out, void* y,
                                       float* rstd, int64_t rows, int d, float eps, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ZS_REQUIRE(x && weight && y, ZS_ERR_ARG);
  ZS_REQUIRE(rows >= 0 && addnorm_nv_ok(d), ZS_ERR_SHAPE);
  ZS_REQUIRE(((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(r) | reinterpret_cast<uintptr_t>(weight) |
               reinterpret_cast<uintptr_t>(h_out) | reinterpret_cast<uintptr_t>(y)) & 15) == 0,
             ZS_ERR_ALIGN);
  ZS_BIND(x);
  if (rows == 0) return ZS_OK;
  switch (d / 128) {
    case 1: return launch_add_zrmsnorm_fwd<1>(x, r, weight, h_out, y, rstd, rows, eps, stream);
    case 2: return launch_add_zrmsnorm_fwd<2>(x, r, weight, h_out, y, rstd, rows, eps, stream);
    case 4: return launch_add_zrmsnorm_fwd<4>(x, r, weight, h_out, y, rstd, rows, eps, stream);
    case 8: return launch_add_zrmsnorm_fwd<8>(x, r, weight, h_out, y, rstd, rows, eps, stream);
    case 12: return launch_add_zrmsnorm_fwd<12>(x, r, weight, h_out, y, rstd, rows, eps, stream);
    default: return launch_add_zrmsnorm_fwd<16>(x, r, weight, h_out, y, rstd, rows, eps, stream);
  }
}

extern "C" int zs_add_zrmsnorm_backward(const void* dy, const float* h, const float* weight, const float* rstd,
                                        const float* dh_in, float* dx, void* dr, float* dweight, int64_t rows, int d,
                                        void* workspace, size_t workspace_bytes, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ZS_REQUIRE(dy && h && weight && rstd && dx && dweight, ZS_ERR_ARG);
  ZS_REQUIRE(rows >= 0 && addnorm_nv_ok(d), ZS_ERR_SHAPE);
  ZS_REQUIRE(workspace && workspace_bytes >= zs_zrmsnorm_backward_workspace(rows, d), ZS_ERR_WORKSPACE);
  ZS_REQUIRE(((reinterpret_cast<uintptr_t>(dy) | reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(dh_in) |
               reinterpret_cast<uintptr_t>(dx) | reinterpret_cast<uintptr_t>(dr)) & 15) == 0,
             ZS_ERR_ALIGN);
  ZS_BIND(h);
  int64_t blocks = (rows + 7) / 8;
  if (blocks > 296) blocks = 296;
  if (blocks < 1) blocks = 1;
  float* part = reinterpret_cast<float*>(workspace);
  int rc;
  switch (d / 128) {
    case 1: rc = launch_add_zrmsnorm_bwd<1>(dy, h, weight, rstd, dh_in, dx, dr, part, blocks, rows, stream); break;
    case 2: rc = launch_add_zrmsnorm_bwd<2>(dy, h, weight, rstd, dh_in, dx, dr, part, blocks, rows, stream); break;
    case 4: rc = launch_add_zrmsnorm_bwd<4>(dy, h, weight, rstd, dh_in, dx, dr, part, blocks, rows, stream); break;
    case 8: rc = launch_add_zrmsnorm_bwd<8>(dy, h, weight, rstd, dh_in, dx, dr, part, blocks, rows, stream); break;
    case 12: rc = launch_add_zrmsnorm_bwd<12>(dy, h, weight, rstd, dh_in, dx, dr, part, blocks, rows, stream); break;
    default: rc = launch_add_zrmsnorm_bwd<16>(dy, h, weight, rstd, dh_in, dx, dr, part, blocks, rows, stream); break;
  }
  if (rc != ZS_OK) return rc;
  if (rows > 0) {
    sum_rows_kernel<<<(d + 255) / 256, 256, 0, stream>>>(part, (int)blocks, d, dweight);
    ZS_CUDA_TRY(cudaGetLastError());
  } else {
    ZS_CUDA_TRY(cudaMemsetAsync(dweight, 0, (size_t)d * sizeof(float), stream));
  }
  return ZS_OK;
}

extern "C" int zs_rope_partial(void* q, int64_t q_row_stride, void* k, int64_t k_row_stride, const void* q_cos,
                               const void* q_sin, const void* k_cos, const void* k_sin, int64_t cos_row_stride,
                               int batch, int seq_len, int cos_batch, int n_q_heads, int n_kv_heads, int head_dim,
                               int rot_pairs, int dtype, int table_dtype, int backward, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ZS_REQUIRE(q && k && q_cos && q_sin && k_cos && k_sin, ZS_ERR_ARG);
  ZS_REQUIRE(batch >= 0 && seq_len >= 1 && n_q_heads >= 1 && n_kv_heads >= 1 && head_dim >= 2 && head_dim % 2 == 0,
             ZS_ERR_SHAPE);
  ZS_REQUIRE(rot_pairs >= 0 && rot_pairs <= head_dim / 2, ZS_ERR_SHAPE);
  if (rot_pairs == 0) return ZS_OK;
  ZS_REQUIRE(cos_batch == 1 || cos_batch == batch, ZS_ERR_SHAPE);
  ZS_BIND(q);
  const int64_t rows = (int64_t)batch * seq_len;
  if (rows == 0) return ZS_OK;
  int64_t blocks = rows < 148 * 32 ? rows : 148 * 32;
  const int threads = 128;
#define ZS_ROPE(T, C)                                                                                            \
  rope_kernel<T, C><<<(unsigned)blocks, threads, 0, stream>>>(                                                 \
      reinterpret_cast<T*>(q), q_row_stride, reinterpret_cast<T*>(k), k_row_stride,                            \
      reinterpret_cast<const C*>(q_cos), reinterpret_cast<const C*>(q_sin), reinterpret_cast<const C*>(k_cos), \
      reinterpret_cast<const C*>(k_sin), cos_row_stride, rows, seq_len, cos_batch, n_q_heads, n_kv_heads,      \
      head_dim, backward, rot_pairs)
  if (dtype == ZS_BF16 && table_dtype == ZS_F32)
    ZS_ROPE(__nv_bfloat16, float);
  else if (dtype == ZS_BF16 && table_dtype == ZS_BF16)
    ZS_ROPE(__nv_bfloat16, __nv_bfloat16);
  else if (dtype == ZS_F32 && table_dtype == ZS_F32)
    ZS_ROPE(float, float);
  else if (dtype == ZS_F16 && table_dtype == ZS_F32)
    ZS_ROPE(__half, float);
  else
    return ZS_ERR_DTYPE;
#undef ZS_ROPE
  ZS_CUDA_TRY(cudaGetLastError());
  return ZS_OK;
}

extern "C" int zs_rope(void* q, int64_t q_row_stride, void* k, int64_t k_row_stride, const void* q_cos,
                       const void* q_sin, const void* k_cos, const void* k_sin, int64_t cos_row_stride, int batch,
                       int seq_len, int cos_batch, int n_q_heads, int n_kv_heads, int head_dim, int dtype,
                       int table_dtype, int backward, void* stream) {
  return zs_rope_partial(q, q_row_stride, k, k_row_stride, q_cos, q_sin, k_cos, k_sin, cos_row_stride, batch,
                         seq_len, cos_batch, n_q_heads, n_kv_heads, head_dim, head_dim / 2, dtype, table_dtype,
                         backward, stream);
}

// ------------------------------------------------------------- q/k norm + RoPE
//
// GatedAttention's per-head QK normalisation followed by its partial position
// RoPE (modeling/attention.py:140-150 with modeling/zRMSNorm.py:4-20 and the
// rotate-half RoPE of modeling/liger_rope.py), fused: one warp per (token,
// head) row of hd values, lane l holding the E = hd/32 consecutive values
// [l*E, l*E + E).  The pair partner of value c (c + hd/2, or c - hd/2) sits in
// lane l ^ 16, one shuffle away.  Rows are the q heads then the k heads of a
// token, read from the leading (Hq + Hk) * hd columns of x (the fused q/k/v/gate
// projection, row stride ldx) and written in the same order to y.  The
// normalised value is rotated in f32 and rounded to bf16 once.
namespace zs {
namespace qkn {

struct Args {
  const __nv_bfloat16* x;
  int64_t ldx;
  const float* wq;
  const float* wk;
  const void* cos;
  const void* sin;
  int table_f32;
  int64_t cos_row_stride;
  int cos_bs;
  int rot;
  int64_t tokens;
  int seq_len, Hq, Hk;
  float eps;
};

template <int E>
__device__ __forceinline__ void load_row(const __nv_bfloat16* p, float (&v)[E]) {
  if constexpr (E == 4) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
  } else {
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
    v[0] = a.x; v[1] = a.y;
  }
}

template <int E>
__device__ __forceinline__ void store_row(__nv_bfloat16* p, const float (&v)[E]) {
  if constexpr (E == 4) {
    __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]), b = __floats2bfloat162_rn(v[2], v[3]);
    *reinterpret_cast<uint2*>(p) = make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
  } else {
    *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(v[0], v[1]);
  }
}

__device__ __forceinline__ float table_at(const Args& a, const void* t, int64_t i) {
  return a.table_f32 ? __ldg(reinterpret_cast<const float*>(t) + i)
                     : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(t)[i]);
}

// rotate the row's values in place: forward (sign +1) x1' = x1 c - x2 s, x2' = x2 c + x1 s;
// backward (sign -1) the transpose.  Lanes below 16 hold the first half of the row.
template <int E>
__device__ __forceinline__ void rotate(const Args& a, int64_t tok, float (&v)[E], float sign) {
  const int lane = threadIdx.x & 31;
  float pv[E];
#pragma unroll
  for (int e = 0; e < E; ++e) pv[e] = __shfl_xor_sync(0xffffffffu, v[e], 16);
  const int p0 = (lane & 15) * E;   // pair index of this lane's first value
  if (p0 >= a.rot) return;
  const int64_t b = tok / a.seq_len, s = tok - b * a.seq_len;
  const int64_t crow = (a.cos_bs == 1 ? s : b * a.seq_len + s) * a.cos_row_stride;
  const bool low = lane < 16;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int p = p0 + e;
    if (p >= a.rot) break;
    const float c = table_at(a, a.cos, crow + p), sn = sign * table_at(a, a.sin, crow + p);
    v[e] = low ? v[e] * c - pv[e] * sn : v[e] * c + pv[e] * sn;
  }
}

template <int E>
__global__ void __launch_bounds__(256) qk_norm_rope_fwd_kernel(Args a, __nv_bfloat16* __restrict__ y, int64_t ldy,
                                                               float* __restrict__ rstd) {
  constexpr int HD = 32 * E;
  const int lane = threadIdx.x & 31;
  const int heads = a.Hq + a.Hk;
  const int64_t rows = a.tokens * heads;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const int64_t tok = r / heads;
    const int hh = (int)(r - tok * heads);
    const float* w = hh < a.Hq ? a.wq : a.wk;
    float v[E];
    load_row<E>(a.x + tok * a.ldx + (int64_t)hh * HD + lane * E, v);
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) ss = fmaf(v[e], v[e], ss);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float rs = rsqrtf(ss / (float)HD + a.eps);
    if (lane == 0) rstd[r] = rs;
#pragma unroll
    for (int e = 0; e < E; ++e) v[e] = (v[e] * rs) * (1.0f + __ldg(w + lane * E + e));
    rotate<E>(a, tok, v, 1.f);
    store_row<E>(y + tok * ldy + (int64_t)hh * HD + lane * E, v);
  }
}

// g = the RoPE transpose of dy; dx = rs * (g (1 + w) - n * mean(g (1 + w) n)), n = x rs;
// dw partial sums (q rows and k rows apart) per block, reduced in a fixed order afterwards.
template <int E>
__global__ void __launch_bounds__(256) qk_norm_rope_bwd_kernel(Args a, const __nv_bfloat16* __restrict__ dy,
                                                               int64_t lddy, const float* __restrict__ rstd,
                                                               __nv_bfloat16* __restrict__ dx, int64_t lddx,
                                                               float* __restrict__ part) {
  constexpr int HD = 32 * E;
  __shared__ float s_acc[8][2][HD];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int heads = a.Hq + a.Hk;
  const int64_t rows = a.tokens * heads;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  float accq[E], acck[E];
#pragma unroll
  for (int e = 0; e < E; ++e) accq[e] = acck[e] = 0.f;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp; r < rows; r += warps) {
    const int64_t tok = r / heads;
    const int hh = (int)(r - tok * heads);
    const bool isq = hh < a.Hq;
    const float* w = isq ? a.wq : a.wk;
    float g[E], xv[E];
    load_row<E>(dy + tok * lddy + (int64_t)hh * HD + lane * E, g);
    load_row<E>(a.x + tok * a.ldx + (int64_t)hh * HD + lane * E, xv);
    rotate<E>(a, tok, g, -1.f);
    const float rs = __ldg(rstd + r);
    float dot = 0.f, dn[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float n = xv[e] * rs;
      dn[e] = g[e] * (1.0f + __ldg(w + lane * E + e));
      dot = fmaf(dn[e], n, dot);
      if (isq) accq[e] = fmaf(g[e], n, accq[e]); else acck[e] = fmaf(g[e], n, acck[e]);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
    const float mean = dot / (float)HD;
    float o[E];
#pragma unroll
    for (int e = 0; e < E; ++e) o[e] = rs * (dn[e] - xv[e] * rs * mean);
    store_row<E>(dx + tok * lddx + (int64_t)hh * HD + lane * E, o);
  }
#pragma unroll
  for (int e = 0; e < E; ++e) {
    s_acc[warp][0][lane * E + e] = accq[e];
    s_acc[warp][1][lane * E + e] = acck[e];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 2 * HD; i += blockDim.x) {
    float t = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) t += s_acc[q][i / HD][i % HD];
    part[(int64_t)blockIdx.x * 2 * HD + i] = t;
  }
}

__global__ void qk_norm_dw_finish_kernel(const float* __restrict__ part, int blocks, int hd, float* __restrict__ dwq,
                                         float* __restrict__ dwk) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 2 * hd) return;
  float t = 0.f;
  for (int b = 0; b < blocks; ++b) t += part[(int64_t)b * 2 * hd + i];
  if (i < hd) dwq[i] = t; else dwk[i - hd] = t;
}

constexpr int BWD_BLOCKS = 148 * 4;

}  // namespace qkn
}  // namespace zs

static int qkn_args(zs::qkn::Args& a, const void* x, int64_t ldx, const float* wq, const float* wk, const void* cos,
                    const void* sin, int table_dtype, int64_t cos_row_stride, int cos_bs, int rot, int64_t tokens,
                    int seq_len, int Hq, int Hk, int hd, float eps) {
  ZS_REQUIRE(x && wq && wk, ZS_ERR_ARG);
  ZS_REQUIRE(hd == 64 || hd == 128, ZS_ERR_SHAPE);
  ZS_REQUIRE(tokens >= 1 && seq_len >= 1 && tokens % seq_len == 0 && Hq >= 1 && Hk >= 1, ZS_ERR_SHAPE);
  ZS_REQUIRE(rot >= 0 && rot <= hd / 2 && (rot == 0 || (cos && sin && cos_bs >= 1)), ZS_ERR_ARG);
  ZS_REQUIRE(table_dtype == ZS_F32 || table_dtype == ZS_BF16, ZS_ERR_DTYPE);
  ZS_REQUIRE(ldx >= (int64_t)(Hq + Hk) * hd && ldx % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 7) == 0,
             ZS_ERR_ALIGN);
  a = zs::qkn::Args{reinterpret_cast<const __nv_bfloat16*>(x), ldx, wq, wk, cos, sin, table_dtype == ZS_F32,
                    cos_row_stride, cos_bs, rot, tokens, seq_len, Hq, Hk, eps};
  return ZS_OK;
}

extern "C" int zs_qk_norm_rope_forward(const void* x, int64_t ldx, const float* wq, const float* wk, const void* cos,
                                       const void* sin, int table_dtype, int64_t cos_row_stride, int cos_bs, int rot,
                                       void* y, int64_t ldy, float* rstd, int64_t tokens, int seq_len, int Hq, int Hk,
                                       int hd, float eps, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  zs::qkn::Args a;
  int rc = qkn_args(a, x, ldx, wq, wk, cos, sin, table_dtype, cos_row_stride, cos_bs, rot, tokens, seq_len, Hq, Hk,
                    hd, eps);
  if (rc != ZS_OK) return rc;
  ZS_REQUIRE(y && rstd, ZS_ERR_ARG);
  ZS_REQUIRE(ldy >= (int64_t)(Hq + Hk) * hd && ldy % 4 == 0 && (reinterpret_cast<uintptr_t>(y) & 7) == 0,
             ZS_ERR_ALIGN);
  ZS_BIND(x);
  const int64_t rows = tokens * (Hq + Hk);
  int64_t blocks = (rows + 7) / 8;
  if (blocks > 148 * 16) blocks = 148 * 16;
  auto* yo = reinterpret_cast<__nv_bfloat16*>(y);
  if (hd == 128)
    zs::qkn::qk_norm_rope_fwd_kernel<4><<<(unsigned)blocks, 256, 0, stream>>>(a, yo, ldy, rstd);
  else
    zs::qkn::qk_norm_rope_fwd_kernel<2><<<(unsigned)blocks, 256, 0, stream>>>(a, yo, ldy, rstd);
  ZS_CUDA_TRY(cudaGetLastError());
  return ZS_OK;
}

extern "C" size_t zs_qk_norm_rope_backward_workspace(int hd) {
  return (size_t)zs::qkn::BWD_BLOCKS * 2 * hd * sizeof(float) + 256;
}

extern "C" int zs_qk_norm_rope_backward(const void* dy, int64_t lddy, const void* x, int64_t ldx, const float* wq,
                                        const float* wk, const void* cos, const void* sin, int table_dtype,
                                        int64_t cos_row_stride, int cos_bs, int rot, const float* rstd, void* dx,
                                        int64_t lddx, float* dwq, float* dwk, int64_t tokens, int seq_len, int Hq,
                                        int Hk, int hd, void* workspace, size_t workspace_bytes, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  zs::qkn::Args a;
  int rc = qkn_args(a, x, ldx, wq, wk, cos, sin, table_dtype, cos_row_stride, cos_bs, rot, tokens, seq_len, Hq, Hk,
                    hd, 0.f);
  if (rc != ZS_OK) return rc;
  ZS_REQUIRE(dy && rstd && dx && dwq && dwk, ZS_ERR_ARG);
  ZS_REQUIRE(lddy >= (int64_t)(Hq + Hk) * hd && lddy % 4 == 0 && (reinterpret_cast<uintptr_t>(dy) & 7) == 0 &&
                 lddx >= (int64_t)(Hq + Hk) * hd && lddx % 4 == 0 && (reinterpret_cast<uintptr_t>(dx) & 7) == 0,
             ZS_ERR_ALIGN);
  ZS_REQUIRE(workspace && workspace_bytes >= zs_qk_norm_rope_backward_workspace(hd), ZS_ERR_WORKSPACE);
  ZS_BIND(x);
  float* part = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  const int blocks = zs::qkn::BWD_BLOCKS;
  const auto* dyi = reinterpret_cast<const __nv_bfloat16*>(dy);
  auto* dxo = reinterpret_cast<__nv_bfloat16*>(dx);
  if (hd == 128)
    zs::qkn::qk_norm_rope_bwd_kernel<4><<<blocks, 256, 0, stream>>>(a, dyi, lddy, rstd, dxo, lddx, part);
  else
    zs::qkn::qk_norm_rope_bwd_kernel<2><<<blocks, 256, 0, stream>>>(a, dyi, lddy, rstd, dxo, lddx, part);
  ZS_CUDA_TRY(cudaGetLastError());
  zs::qkn::qk_norm_dw_finish_kernel<<<(2 * hd + 127) / 128, 128, 0, stream>>>(part, blocks, hd, dwq, dwk);
  ZS_CUDA_TRY(cudaGetLastError());
  return ZS_OK;
}
