// Bandwidth-bound helpers of the scattermoe expert layer: row gather with an
// optional per-row coefficient (group), the gate-gradient row dot product
// (rowwise_sum_product), per-expert column sums (the bias gradient of
// groupXtY) and the k-way weighted row combine that closes the expert layer.
// All are warp-per-row kernels with 16-byte vector accesses when the rows
// allow it; accumulation is f32.
#include "zs_common.cuh"

namespace zs {

__device__ __forceinline__ float load_as_f32(const void* p, int64_t i, int dtype) {
  if (dtype == ZS_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dtype == ZS_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ void store_from_f32(void* p, int64_t i, int dtype, float v) {
  if (dtype == ZS_BF16)
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else if (dtype == ZS_F16)
    reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  else
    reinterpret_cast<float*>(p)[i] = v;
}

// 8 x 16-bit values <-> f32
__device__ __forceinline__ void unpack8(const uint4& w, int dtype, float (&f)[8]) {
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    if (dtype == ZS_F16) {
      __half2 h = *reinterpret_cast<const __half2*>(&u[q]);
      float2 v = __half22float2(h);
      f[2 * q] = v.x;
      f[2 * q + 1] = v.y;
    } else {
      __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&u[q]);
      float2 v = __bfloat1622float2(h);
      f[2 * q] = v.x;
      f[2 * q + 1] = v.y;
    }
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8], int dtype) {
  uint32_t u[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    if (dtype == ZS_F16) {
      __half2 h = __floats2half2_rn(f[2 * q], f[2 * q + 1]);
      u[q] = *reinterpret_cast<uint32_t*>(&h);
    } else {
      __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * q], f[2 * q + 1]);
      u[q] = *reinterpret_cast<uint32_t*>(&h);
    }
  }
  return make_uint4(u[0], u[1], u[2], u[3]);
}

// Y[i] = A[ssi[i] / fan_out] (* coeff[ssi[i]]), one warp per row.
__global__ void group_kernel(const char* A, int64_t a_sm, int64_t K, char* Y, int64_t y_sm, int64_t n,
                             const void* coeff, int coeff_dtype, int fan_out, const int64_t* ssi, int dtype,
                             int vec) {
  const int es = dtype == ZS_F32 ? 4 : 2;
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t i = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < n; i += warps) {
    const int64_t src = __ldg(ssi + i);
    if (src < 0 || src >= n) {
      if (lane == 0) record_error(ZS_DEVERR_INDEX);
      continue;
    }
    const float c = coeff ? load_as_f32(coeff, src, coeff_dtype) : 1.0f;
    const char* srow = A + (src / fan_out) * a_sm * es;
    char* drow = Y + i * y_sm * es;
    if (vec) {
      // four 16-byte vectors per lane in flight before any is stored
      const int64_t nv = K * es / 16;
      for (int64_t v0 = 0; v0 < nv; v0 += 128) {
        uint4 w[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int64_t v = v0 + u * 32 + lane;
          if (v < nv) w[u] = __ldg(reinterpret_cast<const uint4*>(srow) + v);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int64_t v = v0 + u * 32 + lane;
          if (v >= nv) continue;
          if (coeff != nullptr) {
            if (dtype == ZS_F32) {
              float* f = reinterpret_cast<float*>(&w[u]);
              for (int q = 0; q < 4; ++q) f[q] *= c;
            } else {
              float f[8];
              unpack8(w[u], dtype, f);
#pragma unroll
              for (int q = 0; q < 8; ++q) f[q] *= c;
              w[u] = pack8(f, dtype);
            }
          }
          reinterpret_cast<uint4*>(drow)[v] = w[u];
        }
      }
    } else {
      for (int64_t k = lane; k < K; k += 32) {
        float v = load_as_f32(srow, k, dtype);
        if (coeff != nullptr) v *= c;
        store_from_f32(drow, k, dtype, v);
      }
    }
  }
}

int launch_group(const void* A, int64_t a_sm, int64_t K, void* Y, int64_t y_sm, int64_t n, const void* coeff,
                 int coeff_dtype, int fan_out, const int64_t* ssi, int dtype, cudaStream_t stream) {
  if (n == 0 || K == 0) return ZS_OK;
  const int es = dtype == ZS_F32 ? 4 : 2;
  const int vec = ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(Y)) % 16 == 0) &&
                  (K * es) % 16 == 0 && (a_sm * es) % 16 == 0 && (y_sm * es) % 16 == 0;
  const int threads = 256;
  int64_t blocks = (n + 7) / 8;
  if (blocks > 148 * 16) blocks = 148 * 16;
  group_kernel<<<(unsigned)blocks, threads, 0, stream>>>(reinterpret_cast<const char*>(A), a_sm, K,
                                                         reinterpret_cast<char*>(Y), y_sm, n, coeff, coeff_dtype,
                                                         fan_out, ssi, dtype, vec);
  return cudaGetLastError() == cudaSuccess ? ZS_OK : ZS_ERR_CUDA;
}

// Db[e, c] = sum over rows of expert e of DY[r, c]
__global__ void colsum_per_expert_kernel(char* Db, int64_t db_se, int64_t db_sn, const char* DY, int64_t dy_sm,
                                         int64_t N, const int64_t* offs, int dtype) {
  const int e = blockIdx.y;
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= N) return;
  const int64_t r0 = e == 0 ? 0 : offs[e - 1];
  const int64_t r1 = offs[e];
  float acc = 0.f;
  for (int64_t r = r0; r < r1; ++r) acc += load_as_f32(DY, r * dy_sm + c, dtype);
  store_from_f32(Db, e * db_se + c * db_sn, dtype, acc);
}

int launch_colsum_per_expert(void* Db, int64_t db_se, int64_t db_sn, const void* DY, int64_t dy_sm, int64_t N,
                             int num_experts, const int64_t* expert_offsets, int dtype, cudaStream_t stream) {
  dim3 grid((unsigned)((N + 127) / 128), (unsigned)num_experts);
  colsum_per_expert_kernel<<<grid, 128, 0, stream>>>(reinterpret_cast<char*>(Db), db_se, db_sn,
                                                     reinterpret_cast<const char*>(DY), dy_sm, N, expert_offsets,
                                                     dtype);
  return cudaGetLastError() == cudaSuccess ? ZS_OK : ZS_ERR_CUDA;
}

// out[t, f] = sum_h A[t, f, h] * B[t, h]; one warp per (t, f).
__global__ void rowwise_sum_product_kernel(char* out, int out_dtype, int64_t o_s0, int64_t o_s1, const char* A,
                                           int a_dtype, int64_t a_s0, int64_t a_s1, int64_t a_s2, const char* B,
                                           int b_dtype, int64_t b_s0, int64_t b_s1, int64_t T, int64_t F,
                                           int64_t H, int vec) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < T * F; w += warps) {
    const int64_t t = w / F, f = w - t * F;
    float acc = 0.f;
    if (vec) {
      const uint4* pa = reinterpret_cast<const uint4*>(A + (t * a_s0 + f * a_s1) * 2);
      const uint4* pb = reinterpret_cast<const uint4*>(B + (t * b_s0) * 2);
      // four vectors of each operand per lane in flight before the products
      for (int64_t v0 = 0; v0 < H / 8; v0 += 128) {
        uint4 ra[4], rb[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int64_t v = v0 + u * 32 + lane;
          if (v < H / 8) {
            ra[u] = __ldg(pa + v);
            rb[u] = __ldg(pb + v);
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (v0 + u * 32 + lane >= H / 8) continue;
          float fa[8], fb[8];
          unpack8(ra[u], a_dtype, fa);
          unpack8(rb[u], b_dtype, fb);
#pragma unroll
          for (int q = 0; q < 8; ++q) acc = fmaf(fa[q], fb[q], acc);
        }
      }
    } else {
      for (int64_t h = lane; h < H; h += 32)
        acc = fmaf(load_as_f32(A, t * a_s0 + f * a_s1 + h * a_s2, a_dtype), load_as_f32(B, t * b_s0 + h * b_s1, b_dtype),
                   acc);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) store_from_f32(out, t * o_s0 + f * o_s1, out_dtype, acc);
  }
}

// out[t, c] = sum_j w[t, j] * in[t*k + j, c]   (w == NULL: plain sum over j)
// f32 accumulation; one warp per token row, 8 columns per lane step.
// rmap (optional, [T*k]): slot t*k+j reads input row rmap[t*k+j] instead of t*k+j
// (rows stored in another order); a row outside [0, n_rows) counts as zero and
// records ZS_DEVERR_INDEX.
__global__ void weighted_row_sum_kernel(char* out, int64_t o_sm, const char* in, int64_t i_sm, const void* w,
                                        int w_dtype, int64_t T, int k, int64_t C, int dtype, int vec,
                                        const int64_t* __restrict__ rmap, int64_t n_rows) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T; t += warps) {
    float wt[32];
    int64_t rw[32];
    for (int j = 0; j < k; ++j) {
      wt[j] = w ? load_as_f32(w, t * k + j, w_dtype) : 1.0f;
      int64_t r = t * k + j;
      if (rmap != nullptr) {
        r = __ldg(rmap + t * k + j);
        if (r < 0 || r >= n_rows) {
          if (lane == 0) zs::record_error(ZS_DEVERR_INDEX);
          r = -1;
        }
      }
      if (r < 0) {
        wt[j] = 0.f;   // contributes nothing; row 0 keeps the load in bounds
        r = 0;
      }
      rw[j] = r;
    }
    if (vec && k <= 8) {
      // all k slot rows' vectors in flight before the accumulation (same j order)
      for (int64_t v = lane; v < C / 8; v += 32) {
        uint4 raw[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (j < k) raw[j] = __ldg(reinterpret_cast<const uint4*>(in + (rw[j] * i_sm) * 2) + v);
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (j >= k) break;
          float f[8];
          unpack8(raw[j], dtype, f);
#pragma unroll
          for (int q = 0; q < 8; ++q) acc[q] = fmaf(wt[j], f[q], acc[q]);
        }
        reinterpret_cast<uint4*>(out + (t * o_sm) * 2)[v] = pack8(acc, dtype);
      }
    } else if (vec) {
      for (int64_t v = lane; v < C / 8; v += 32) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int j = 0; j < k; ++j) {
          float f[8];
          unpack8(__ldg(reinterpret_cast<const uint4*>(in + (rw[j] * i_sm) * 2) + v), dtype, f);
#pragma unroll
          for (int q = 0; q < 8; ++q) acc[q] = fmaf(wt[j], f[q], acc[q]);
        }
        reinterpret_cast<uint4*>(out + (t * o_sm) * 2)[v] = pack8(acc, dtype);
      }
    } else {
      for (int64_t c = lane; c < C; c += 32) {
        float acc = 0.f;
        for (int j = 0; j < k; ++j) acc = fmaf(wt[j], load_as_f32(in, rw[j] * i_sm + c, dtype), acc);
        store_from_f32(out, t * o_sm + c, dtype, acc);
      }
    }
  }
}

}  // namespace zs

using namespace zs;

extern "C" int zs_group(const void* A, int64_t a_sm, int64_t K, void* Y, int64_t y_sm, int64_t n, const void* coeff,
                        int coeff_dtype, int fan_out, const int64_t* sorted_scattered_idxs, int dtype, void* stream) {
  ZS_REQUIRE(A && Y && sorted_scattered_idxs, ZS_ERR_ARG);
  ZS_REQUIRE(dtype == ZS_BF16 || dtype == ZS_F16 || dtype == ZS_F32, ZS_ERR_DTYPE);
  ZS_REQUIRE(coeff == nullptr || coeff_dtype == ZS_BF16 || coeff_dtype == ZS_F16 || coeff_dtype == ZS_F32,
             ZS_ERR_DTYPE);
  ZS_REQUIRE(K >= 0 && n >= 0 && fan_out >= 1, ZS_ERR_SHAPE);
  ZS_BIND(A);
  return launch_group(A, a_sm, K, Y, y_sm, n, coeff, coeff_dtype, fan_out, sorted_scattered_idxs, dtype,
                      static_cast<cudaStream_t>(stream));
}

extern "C" int zs_rowwise_sum_product(void* out, int out_dtype, int64_t o_s0, int64_t o_s1, const void* A,
                                      int a_dtype, int64_t a_s0, int64_t a_s1, int64_t a_s2, const void* B,
                                      int b_dtype, int64_t b_s0, int64_t b_s1, int64_t T, int64_t F, int64_t H,
                                      void* stream) {
  ZS_REQUIRE(out && A && B, ZS_ERR_ARG);
  ZS_REQUIRE(T >= 0 && F >= 0 && H >= 0, ZS_ERR_SHAPE);
  ZS_BIND(A);
  if (T * F == 0) return ZS_OK;
  const int vec = a_dtype != ZS_F32 && b_dtype != ZS_F32 && a_s2 == 1 && b_s1 == 1 && H % 8 == 0 &&
                  (a_s0 % 8 == 0) && (a_s1 % 8 == 0) && (b_s0 % 8 == 0) &&
                  ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) % 16 == 0);
  int64_t blocks = (T * F + 7) / 8;
  if (blocks > 148 * 16) blocks = 148 * 16;
  rowwise_sum_product_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<char*>(out), out_dtype, o_s0, o_s1, reinterpret_cast<const char*>(A), a_dtype, a_s0, a_s1, a_s2,
      reinterpret_cast<const char*>(B), b_dtype, b_s0, b_s1, T, F, H, vec);
  return cudaGetLastError() == cudaSuccess ? ZS_OK : ZS_ERR_CUDA;
}

extern "C" int zs_weighted_row_sum(void* out, int64_t o_sm, const void* in, int64_t i_sm, const void* weights,
                                   int w_dtype, int64_t T, int k, int64_t C, int dtype, void* stream) {
  ZS_REQUIRE(out && in, ZS_ERR_ARG);
  ZS_REQUIRE(dtype == ZS_BF16 || dtype == ZS_F16, ZS_ERR_DTYPE);
  ZS_REQUIRE(T >= 0 && k >= 1 && k <= 32 && C >= 0, ZS_ERR_SHAPE);
  ZS_BIND(in);
  if (T == 0 || C == 0) return ZS_OK;
  const int vec = C % 8 == 0 && o_sm % 8 == 0 && i_sm % 8 == 0 &&
                  ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(in)) % 16 == 0);
  int64_t blocks = (T + 7) / 8;
  if (blocks > 148 * 16) blocks = 148 * 16;
  weighted_row_sum_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<char*>(out), o_sm, reinterpret_cast<const char*>(in), i_sm, weights, w_dtype, T, k, C, dtype,
      vec, nullptr, T * k);
  return cudaGetLastError() == cudaSuccess ? ZS_OK : ZS_ERR_CUDA;
}

namespace zs {
// The MoE layer's output added into the f32 residual stream in one pass:
//   out[t] = residual[t] + (f32(shared[t]) + f32(bf16(sum_j w[t, j] * rows[t*k + j])))
// -- the values of the block's `h + (shared.float() + routed)` with the routed
// combine rounded to the storage dtype first, as the unfused path computes them.
// rows / shared in dtype (bf16 or f16), residual / out f32; C % 8 == 0.
__global__ void moe_combine_kernel(float* __restrict__ out, int64_t o_sm, const char* __restrict__ in, int64_t i_sm,
                                   const void* w, int w_dtype, int64_t T, int k, int64_t C, int dtype,
                                   const char* __restrict__ shared, int64_t s_sm, const float* __restrict__ residual,
                                   int64_t r_sm) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T; t += warps) {
    float wt[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) wt[j] = (j < k && w != nullptr) ? load_as_f32(w, t * k + j, w_dtype) : 1.0f;
    for (int64_t v = lane; v < C / 8; v += 32) {
      uint4 raw[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j < k) raw[j] = __ldg(reinterpret_cast<const uint4*>(in + ((t * k + j) * i_sm) * 2) + v);
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (j >= k) break;
        float f[8];
        unpack8(raw[j], dtype, f);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] = fmaf(wt[j], f[q], acc[q]);
      }
      float r8[8];
      unpack8(pack8(acc, dtype), dtype, r8);   // the routed sum in the storage dtype
      if (shared != nullptr) {
        float s8[8];
        unpack8(__ldg(reinterpret_cast<const uint4*>(shared + (t * s_sm) * 2) + v), dtype, s8);
#pragma unroll
        for (int q = 0; q < 8; ++q) r8[q] = s8[q] + r8[q];
      }
      float4* o4 = reinterpret_cast<float4*>(out + t * o_sm) + 2 * v;
      if (residual != nullptr) {
        const float4* x4 = reinterpret_cast<const float4*>(residual + t * r_sm) + 2 * v;
        const float4 a = __ldg(x4), b = __ldg(x4 + 1);
        o4[0] = make_float4(a.x + r8[0], a.y + r8[1], a.z + r8[2], a.w + r8[3]);
        o4[1] = make_float4(b.x + r8[4], b.y + r8[5], b.z + r8[6], b.w + r8[7]);
      } else {
        o4[0] = make_float4(r8[0], r8[1], r8[2], r8[3]);
        o4[1] = make_float4(r8[4], r8[5], r8[6], r8[7]);
      }
    }
  }
}
}  // namespace zs

extern "C" int zs_moe_combine(float* out, int64_t o_sm, const void* rows, int64_t i_sm, const void* weights,
                              int w_dtype, int64_t T, int k, int64_t C, int dtype, const void* shared, int64_t s_sm,
                              const float* residual, int64_t r_sm, void* stream) {
  ZS_REQUIRE(out && rows, ZS_ERR_ARG);
  ZS_REQUIRE(dtype == ZS_BF16 || dtype == ZS_F16, ZS_ERR_DTYPE);
  ZS_REQUIRE(T >= 0 && k >= 1 && k <= 8 && C >= 0, ZS_ERR_SHAPE);
  ZS_REQUIRE(C % 8 == 0 && o_sm % 4 == 0 && i_sm % 8 == 0 && (shared == nullptr || s_sm % 8 == 0) &&
                 (residual == nullptr || r_sm % 4 == 0) &&
                 ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(rows) |
                   reinterpret_cast<uintptr_t>(shared) | reinterpret_cast<uintptr_t>(residual)) % 16 == 0),
             ZS_ERR_ALIGN);
  ZS_BIND(rows);
  if (T == 0 || C == 0) return ZS_OK;
  int64_t blocks = (T + 7) / 8;
  if (blocks > 148 * 16) blocks = 148 * 16;
  zs::moe_combine_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      out, o_sm, reinterpret_cast<const char*>(rows), i_sm, weights, w_dtype, T, k, C, dtype,
      reinterpret_cast<const char*>(shared), s_sm, residual, r_sm);
  return cudaGetLastError() == cudaSuccess ? ZS_OK : ZS_ERR_CUDA;
}

extern "C" int zs_gathered_row_sum(void* out, int64_t o_sm, const void* in, int64_t i_sm, int64_t n_rows,
                                   const int64_t* row_of_slot, int64_t T, int k, int64_t C, int dtype,
                                   void* stream) {
  ZS_REQUIRE(out && in && row_of_slot, ZS_ERR_ARG);
  ZS_REQUIRE(dtype == ZS_BF16 || dtype == ZS_F16, ZS_ERR_DTYPE);
  ZS_REQUIRE(T >= 0 && k >= 1 && k <= 32 && C >= 0 && n_rows >= 0, ZS_ERR_SHAPE);
  ZS_BIND(in);
  if (T == 0 || C == 0) return ZS_OK;
  const int vec = C % 8 == 0 && o_sm % 8 == 0 && i_sm % 8 == 0 &&
                  ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(in)) % 16 == 0);
  int64_t blocks = (T + 7) / 8;
  if (blocks > 148 * 16) blocks = 148 * 16;
  weighted_row_sum_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<char*>(out), o_sm, reinterpret_cast<const char*>(in), i_sm, nullptr, 0, T, k, C, dtype, vec,
      row_of_slot, n_rows);
  return cudaGetLastError() == cudaSuccess ? ZS_OK : ZS_ERR_CUDA;
}

namespace zs {
// Backward of act = silu(g) * h with hfull = [h | g] per row, replaying the
// rounding points of the reference's autograd in the storage dtype:
//   s = silu(g), dh = dact * s, t = dact * h, dg = t * sig * (1 + g * (1 - sig))
template <typename T>
__global__ void swiglu_backward_kernel(T* __restrict__ dhfull, const T* __restrict__ dact, const T* __restrict__ hfull,
                                       int64_t n, int64_t F) {
  const int64_t total = n * F;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / F, c = i - r * F;
    const float da = to_f32<T>(dact[i]);
    const float h = to_f32<T>(hfull[r * 2 * F + c]);
    const float g = to_f32<T>(hfull[r * 2 * F + F + c]);
    const float sig = 1.0f / (1.0f + expf(-g));
    const float s = to_f32<T>(from_f32<T>(g / (1.0f + expf(-g))));
    dhfull[r * 2 * F + c] = from_f32<T>(da * s);
    const float t = to_f32<T>(from_f32<T>(da * h));
    dhfull[r * 2 * F + F + c] = from_f32<T>(t * (sig * (1.0f + g * (1.0f - sig))));
  }
}
}  // namespace zs

extern "C" int zs_swiglu_backward(void* dhfull, const void* dact, const void* hfull, int64_t n, int64_t F, int dtype,
                                  void* stream) {
  ZS_REQUIRE(dhfull && dact && hfull, ZS_ERR_ARG);
  ZS_REQUIRE(n >= 0 && F >= 1, ZS_ERR_SHAPE);
  ZS_BIND(dact);
  if (n == 0) return ZS_OK;
  int64_t blocks = (n * F + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == ZS_BF16)
    swiglu_backward_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, s>>>(
        reinterpret_cast<__nv_bfloat16*>(dhfull), reinterpret_cast<const __nv_bfloat16*>(dact),
        reinterpret_cast<const __nv_bfloat16*>(hfull), n, F);
  else if (dtype == ZS_F16)
    swiglu_backward_kernel<__half><<<(unsigned)blocks, 256, 0, s>>>(reinterpret_cast<__half*>(dhfull),
                                                                     reinterpret_cast<const __half*>(dact),
                                                                     reinterpret_cast<const __half*>(hfull), n, F);
  else if (dtype == ZS_F32)
    swiglu_backward_kernel<float><<<(unsigned)blocks, 256, 0, s>>>(reinterpret_cast<float*>(dhfull),
                                                                   reinterpret_cast<const float*>(dact),
                                                                   reinterpret_cast<const float*>(hfull), n, F);
  else
    return ZS_ERR_DTYPE;
  return cudaGetLastError() == cudaSuccess ? ZS_OK : ZS_ERR_CUDA;
}
