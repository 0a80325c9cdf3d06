// MuonMD bookkeeping around Newton-Schulz (optimizer/muon.py:398-508), fused.
//
// The reference runs the magnitude/direction step as ~40 f32 tensor passes
// over each weight stack W [L, m, n] (the gain outer product is materialised,
// W / g, g * G, the momentum lerps, the projection, the gain reductions ...).
// Here it is three passes over the stack plus one tiny kernel:
//   md_pre_kernel     reads W, G, buf -> writes buf and the bf16 Newton-Schulz
//                     input X = lerp(g*G, buf', momentum); reduces the gain
//                     gradients (W/g)*G over the axes each gain does not span
//   md_reduce_kernel  reads W, U (the orthogonalised update) -> sum of squares
//                     of W_hat' = W/g - lr*rescale*U per matrix / row / column
//   md_gain_kernel    gain Adam steps (softplus chain rule), projection scales
//   md_write_kernel   reads W, U -> p = g_new * W_hat' * target / ||W_hat'||
// Tile: 64 rows x 256 columns per block of 256 threads; warp w owns rows
// w*8 .. w*8+7, lane owns 8 consecutive columns (two float4 per f32 operand).
// Reductions are deterministic: each block writes its partial row / column /
// matrix sums to a scratch slot of its own (no atomics), and md_finish_kernel
// adds the slots in a fixed order.  Every run -- and every data-parallel
// replica -- therefore computes bit-identical gains and projections.
#include <initializer_list>
#include <type_traits>

#include "zs_common.cuh"

namespace zs {
namespace md {

constexpr int TR = 64, TC = 256, THREADS = 256;

__device__ __forceinline__ float softplus_f(float x) { return x > 20.f ? x : log1pf(expf(x)); }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + expf(-x)); }
// torch.lerp's two-sided form
__device__ __forceinline__ float lerp_f(float a, float b, float w) {
  const float d = b - a;
  return w < 0.5f ? a + w * d : b - d * (1.f - w);
}

struct Gains {
  const float* sc;   // raw scalar gain [L] or null
  const float* row;  // raw row gain [L, m] or null
  const float* col;  // raw column gain [L, n] or null
};

// 8 consecutive f32 of a row (vectorised when VEC)
template <bool VEC>
__device__ __forceinline__ void load8(const float* p, int64_t c, int64_t n, float (&v)[8]) {
  if (VEC) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p + c));
    const float4 b = __ldg(reinterpret_cast<const float4*>(p + c + 4));
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = c + e < n ? p[c + e] : 0.f;
  }
}

template <bool VEC>
__device__ __forceinline__ void load8_mut(const float* p, int64_t c, int64_t n, float (&v)[8]) {
  if (VEC) {
    const float4 a = *reinterpret_cast<const float4*>(p + c);
    const float4 b = *reinterpret_cast<const float4*>(p + c + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = c + e < n ? p[c + e] : 0.f;
  }
}

template <bool VEC>
__device__ __forceinline__ void store8(float* p, int64_t c, int64_t n, const float (&v)[8]) {
  if (VEC) {
    *reinterpret_cast<float4*>(p + c) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(p + c + 4) = make_float4(v[4], v[5], v[6], v[7]);
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (c + e < n) p[c + e] = v[e];
  }
}

template <bool VEC>
__device__ __forceinline__ void load8_bf16(const __nv_bfloat16* p, int64_t c, int64_t n, float (&v)[8]) {
  if (VEC) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p + c));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(h[e]);
      v[2 * e] = f.x;
      v[2 * e + 1] = f.y;
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = c + e < n ? __bfloat162float(p[c + e]) : 0.f;
  }
}

// 8 consecutive bf16 of a row as four packed pairs (zeros past n); unpacked by unpack8_bf16
template <bool VEC>
__device__ __forceinline__ void load8_bf16_raw(const __nv_bfloat16* p, int64_t c, int64_t n, uint32_t (&r)[4]) {
  if (VEC) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p + c));
    r[0] = u.x; r[1] = u.y; r[2] = u.z; r[3] = u.w;
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      __nv_bfloat162 h;
      h.x = c + 2 * e < n ? p[c + 2 * e] : __float2bfloat16_rn(0.f);
      h.y = c + 2 * e + 1 < n ? p[c + 2 * e + 1] : __float2bfloat16_rn(0.f);
      r[e] = *reinterpret_cast<uint32_t*>(&h);
    }
  }
}

__device__ __forceinline__ void unpack8_bf16(const uint32_t (&r)[4], float (&v)[8]) {
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r[e]));
    v[2 * e] = f.x;
    v[2 * e + 1] = f.y;
  }
}

template <bool VEC>
__device__ __forceinline__ void store8_bf16(__nv_bfloat16* p, int64_t c, int64_t n, const float (&v)[8]) {
  if (VEC) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
    *reinterpret_cast<uint4*>(p + c) = u;
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (c + e < n) p[c + e] = __float2bfloat16_rn(v[e]);
  }
}

// block-wide sum; every thread gets the result
__device__ __forceinline__ float block_sum(float v, float* sh) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < THREADS / 32; ++w) t += sh[w];
  return t;
}

// softplus'd gains of the tile into shared memory (1 where a gain is absent)
// Also the reciprocals s_ri[i] = 1 / (scalar * row gain) and s_ci[j] = 1 / column gain: the
// passes divide W by the gain product as W * (s_ri * s_ci) (a few ulps from the quotient,
// and a multiply instead of an IEEE division per element).
__device__ __forceinline__ float tile_gains(const Gains& g, int64_t l, int64_t m, int64_t n, int64_t r0, int64_t c0,
                                            float* s_r, float* s_c, float* s_ri, float* s_ci) {
  const float sc = g.sc != nullptr ? softplus_f(g.sc[l]) : 1.f;
  for (int i = threadIdx.x; i < TR; i += THREADS) {
    const float r = (g.row != nullptr && r0 + i < m) ? softplus_f(g.row[l * m + r0 + i]) : 1.f;
    s_r[i] = r;
    s_ri[i] = 1.0f / (sc * r);
  }
  for (int i = threadIdx.x; i < TC; i += THREADS) {
    const float c = (g.col != nullptr && c0 + i < n) ? softplus_f(g.col[l * n + c0 + i]) : 1.f;
    s_c[i] = c;
    s_ci[i] = 1.0f / c;
  }
  return sc;
}

// The vectorised post passes stage each thread's eight rows of W (two 16-byte chunks
// a row) and, in the plain layout, of U (one chunk) into shared memory with
// cp.async before any arithmetic: all of a block's loads are in flight at once
// without holding registers (96 KB a block, two blocks an SM).  Chunk j of row k of
// thread t sits at [(k * NCH + j) * THREADS + t], so a warp's 16-byte reads are
// contiguous.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

template <bool TRANS>
struct Stage {
  static constexpr int NCH = TRANS ? 2 : 3;
  static constexpr int BYTES = 8 * NCH * THREADS * 16;
};

template <bool TRANS>
__device__ __forceinline__ void stage_rows(uint4* st, const float* W, const __nv_bfloat16* U, int64_t l, int64_t m,
                                           int64_t n, int64_t r0, int64_t c) {
  constexpr int NCH = Stage<TRANS>::NCH;
  const int warp = threadIdx.x >> 5, tid = threadIdx.x;
  if (c >= n) return;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int64_t row = r0 + warp * 8 + k;
    if (row >= m) break;
    const int64_t off = (l * m + row) * n + c;
    cp_async16(&st[(k * NCH + 0) * THREADS + tid], W + off);
    cp_async16(&st[(k * NCH + 1) * THREADS + tid], W + off + 4);
    if constexpr (!TRANS) cp_async16(&st[(k * NCH + 2) * THREADS + tid], U + off);
  }
}

__device__ __forceinline__ void staged_w(const uint4* st, int k, int nch, float (&w)[8]) {
  const int tid = threadIdx.x;
  const uint4 a = st[(k * nch + 0) * THREADS + tid], b = st[(k * nch + 1) * THREADS + tid];
  w[0] = __uint_as_float(a.x); w[1] = __uint_as_float(a.y); w[2] = __uint_as_float(a.z); w[3] = __uint_as_float(a.w);
  w[4] = __uint_as_float(b.x); w[5] = __uint_as_float(b.y); w[6] = __uint_as_float(b.z); w[7] = __uint_as_float(b.w);
}

// Transposed bf16 layout [L, n, m] of the Newton-Schulz operand of a tall stack (m > n
// runs as its transpose): a block's 64 x 256 tile is staged in shared memory as 256
// columns of 32 words (row pairs), the word of row pair q of tile column j stored at
// q ^ (j / 8 mod 32) -- a thread's eight columns j = lane*8 + e then fall in 32
// different banks, and a warp moving one column to or from global memory touches each
// bank once with 128 contiguous bytes.
constexpr int TW = TR / 2;   // words per staged column

__device__ __forceinline__ int tswz(int j, int q) { return q ^ ((j >> 3) & 31); }

// global [L, n, m] -> staged tile (zeros outside the matrix); whole row pairs are copied
// with cp.async (the caller waits for them with cp_async_wait_all before its barrier)
__device__ __forceinline__ void stage_t_load(uint32_t (*s_t)[TW], const __nv_bfloat16* __restrict__ T, int64_t l,
                                             int64_t m, int64_t n, int64_t r0, int64_t c0, bool words) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t i = r0 + 2 * lane;
  for (int j = warp; j < TC; j += THREADS / 32) {
    const int64_t col = c0 + j;
    uint32_t* dst = &s_t[j][tswz(j, lane)];
    const __nv_bfloat16* src = T + (l * n + col) * m + i;
    if (col < n && words && i + 1 < m) {
      asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
    } else {
      __nv_bfloat162 h;
      h.x = (col < n && i < m) ? src[0] : __float2bfloat16_rn(0.f);
      h.y = (col < n && i + 1 < m) ? src[1] : __float2bfloat16_rn(0.f);
      *dst = *reinterpret_cast<uint32_t*>(&h);
    }
  }
}

// staged tile -> global [L, n, m] (only elements inside the matrix)
__device__ __forceinline__ void stage_t_store(const uint32_t (*s_t)[TW], __nv_bfloat16* __restrict__ T, int64_t l,
                                              int64_t m, int64_t n, int64_t r0, int64_t c0, bool words) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll 4
  for (int j = warp; j < TC; j += THREADS / 32) {
    const int64_t col = c0 + j;
    if (col >= n) continue;
    const int q = tswz(j, lane);          // this lane's physical word holds logical row pair q
    const uint32_t v = s_t[j][lane];
    const int64_t i = r0 + 2 * q;
    __nv_bfloat16* dst = T + (l * n + col) * m + i;
    if (words && i + 1 < m) {
      *reinterpret_cast<uint32_t*>(dst) = v;
    } else {
      const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&v);
      if (i < m) dst[0] = h.x;
      if (i + 1 < m) dst[1] = h.y;
    }
  }
}

// the eight staged values of tile row rr at columns lane*8 .. lane*8+7, as four bf16 pairs
__device__ __forceinline__ void stage_t_row(const uint32_t (*s_t)[TW], int rr, int lane, uint32_t (&r)[4]) {
  const int sh = (rr & 1) * 16;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const uint32_t lo = (s_t[lane * 8 + 2 * e][(rr >> 1) ^ lane] >> sh) & 0xffffu;
    const uint32_t hi = (s_t[lane * 8 + 2 * e + 1][(rr >> 1) ^ lane] >> sh) & 0xffffu;
    r[e] = lo | (hi << 16);
  }
}

// Pre-Newton-Schulz: buf.lerp_(g*G, 1-mom); X = lerp(g*G, buf, mom) (bf16);
// gain gradients (before the sigmoid factor) from the old gains, as per-block
// partial sums that md_finish_kernel adds up:
//   red_s[l]    = sum (W/g)*G * r*c     red_r[l,i] = sum_j (W/g)*G * c*s
//   red_c[l,j]  = sum_i (W/g)*G * r*s
// Partial sums of one block (bx, by) of matrix l: rows [L, m, gx], columns
// [L, gy, n], whole matrix [L, gy * gx]; md_finish_kernel reduces them.
struct Partials {
  float* r;
  float* c;
  float* s;
};

// TRANS: X is written in the transposed layout [L, n, m] (words: m even and X 4-byte aligned).
template <bool VEC, bool TRANS>
__global__ void __launch_bounds__(THREADS, 2) md_pre_kernel(const float* __restrict__ W, const float* __restrict__ G,
                                                         float* __restrict__ buf, Gains gains,
                                                         __nv_bfloat16* __restrict__ X, Partials part, bool want_s,
                                                         bool want_r, bool want_c, int64_t m, int64_t n, float mom,
                                                         bool words) {
  __shared__ float s_r[TR], s_c[TC], s_ri[TR], s_ci[TC], s_col[THREADS / 32][TC], sh[32];
  __shared__ uint32_t s_t[TRANS ? TC : 1][TW];
  const int64_t l = blockIdx.z, r0 = (int64_t)blockIdx.y * TR, c0 = (int64_t)blockIdx.x * TC;
  const float sc = tile_gains(gains, l, m, n, r0, c0, s_r, s_c, s_ri, s_ci);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool have_g = gains.sc != nullptr || gains.row != nullptr || gains.col != nullptr;
  const int64_t c = c0 + lane * 8;
  float colacc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float sacc = 0.f;
  // four batches of two rows: each batch's six 32-byte loads are issued before its
  // arithmetic and stores (buf is read and written in place, so the compiler keeps the
  // loads of a later row behind an earlier row's stores)
#pragma unroll 1
  for (int kb = 0; kb < 8; kb += 2) {
    float w[2][8], gr[2][8], b[2][8];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int64_t row = r0 + warp * 8 + kb + k;
      if (row < m && c < n) {
        const int64_t off = (l * m + row) * n;
        load8<VEC>(W + off, c, n, w[k]);
        load8<VEC>(G + off, c, n, gr[k]);
        load8_mut<VEC>(buf + off, c, n, b[k]);
      }
    }
    float x[2][8];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int rr = warp * 8 + kb + k;
      const int64_t row = r0 + rr;
#pragma unroll
      for (int e = 0; e < 8; ++e) x[k][e] = 0.f;
      if (row >= m) continue;
      float racc = 0.f;
      if (c < n) {
        const int64_t off = (l * m + row) * n;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float cg = s_c[lane * 8 + e];
          float gh = gr[k][e];
          if (have_g) {
            const float gv = (sc * s_r[rr]) * cg;
            const float wg = (w[k][e] * (s_ri[rr] * s_ci[lane * 8 + e])) * gr[k][e];
            gh = gv * gr[k][e];
            racc += wg * (cg * sc);
            colacc[e] += wg * (s_r[rr] * sc);
            sacc += wg * (s_r[rr] * cg);
          }
          b[k][e] = lerp_f(b[k][e], gh, 1.f - mom);
          x[k][e] = lerp_f(gh, b[k][e], mom);
        }
        store8<VEC>(buf + off, c, n, b[k]);
        if constexpr (!TRANS) store8_bf16<VEC>(X + off, c, n, x[k]);
      }
      if (want_r) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) racc += __shfl_xor_sync(0xffffffffu, racc, o);
        if (lane == 0) part.r[(l * m + row) * gridDim.x + blockIdx.x] = racc;
      }
    }
    if constexpr (TRANS) {
      // rows kb, kb+1 of this warp form row pair (warp*8 + kb) / 2 of every column
      const int q = (warp * 8 + kb) >> 1;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(x[0][e], x[1][e]);
        s_t[lane * 8 + e][q ^ lane] = *reinterpret_cast<const uint32_t*>(&h);
      }
    }
  }
  if constexpr (TRANS) {
    __syncthreads();
    stage_t_store(s_t, X, l, m, n, r0, c0, words);
  }
  if (want_c) {
#pragma unroll
    for (int e = 0; e < 8; ++e) s_col[warp][lane * 8 + e] = colacc[e];
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < THREADS / 32; ++w) t += s_col[w][threadIdx.x];
    if (c0 + threadIdx.x < n) part.c[(l * gridDim.y + blockIdx.y) * n + c0 + threadIdx.x] = t;
  }
  if (want_s) {
    const float t = block_sum(sacc, sh);
    if (threadIdx.x == 0) part.s[l * gridDim.y * gridDim.x + blockIdx.y * gridDim.x + blockIdx.x] = t;
  }
}

// out[i] = sum_{k < K} part[(i / inner) * K * inner + i % inner + k * inner], k ascending:
// rows (inner 1, K = gx), whole matrices (inner 1, K = gy * gx), columns (inner n, K = gy).
__global__ void md_finish_kernel(const float* __restrict__ part, float* __restrict__ out, int64_t count,
                                 int64_t inner, int K) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
    const float* p = part + (i / inner) * K * inner + i % inner;
    float t = 0.f;
    for (int k = 0; k < K; ++k) t += p[k * inner];
    out[i] = t;
  }
}

struct PostArgs {
  const float* W;
  const __nv_bfloat16* U;
  int64_t m, n;
  const float* lr_dev;
  float lr_host;
  float rescale;
  int norm_axis;          // 0 frobenius, 1 row, 2 column
  bool u_words;           // transposed U: m even and U 4-byte aligned (32-bit row-pair accesses)
};

__device__ __forceinline__ float lr_of(const PostArgs& a) { return a.lr_dev != nullptr ? __ldg(a.lr_dev) : a.lr_host; }

// sum of squares of W_hat' = W/g - lr * (rescale * U) per matrix / row / column
// (TRANS: U in the transposed layout [L, n, m])
template <bool VEC, bool TRANS>
__global__ void __launch_bounds__(THREADS, 2) md_reduce_kernel(PostArgs a, Gains gains, Partials part) {
  __shared__ float s_r[TR], s_c[TC], s_ri[TR], s_ci[TC], s_col[THREADS / 32][TC], sh[32];
  __shared__ uint32_t s_t[TRANS ? TC : 1][TW];
  extern __shared__ __align__(16) uint8_t md_dyn[];
  uint4* st = reinterpret_cast<uint4*>(md_dyn);
  const int64_t m = a.m, n = a.n;
  const int64_t l = blockIdx.z, r0 = (int64_t)blockIdx.y * TR, c0 = (int64_t)blockIdx.x * TC;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t c = c0 + lane * 8;
  if constexpr (VEC) stage_rows<TRANS>(st, a.W, a.U, l, m, n, r0, c);
  tile_gains(gains, l, m, n, r0, c0, s_r, s_c, s_ri, s_ci);
  if constexpr (TRANS) stage_t_load(s_t, a.U, l, m, n, r0, c0, a.u_words);
  if constexpr (VEC || TRANS) cp_async_wait_all();
  __syncthreads();
  const float lrr = lr_of(a) * a.rescale;
  float colacc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float facc = 0.f;
#pragma unroll 2
  for (int k = 0; k < 8; ++k) {
    const int rr = warp * 8 + k;
    const int64_t row = r0 + rr;
    // rows past m and columns past n read as zeros and add nothing
    float w[8], u[8];
    uint32_t ur[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int e = 0; e < 8; ++e) w[e] = 0.f;
    if (row < m && c < n) {
      if constexpr (VEC) {
        staged_w(st, k, Stage<TRANS>::NCH, w);
        if constexpr (!TRANS) {
          const uint4 q4 = st[(k * 3 + 2) * THREADS + threadIdx.x];
          ur[0] = q4.x; ur[1] = q4.y; ur[2] = q4.z; ur[3] = q4.w;
        }
      } else {
        load8<VEC>(a.W + (l * m + row) * n, c, n, w);
        if constexpr (!TRANS) load8_bf16_raw<VEC>(a.U + (l * m + row) * n, c, n, ur);
      }
      if constexpr (TRANS) stage_t_row(s_t, rr, lane, ur);
    }
    unpack8_bf16(ur, u);
    float racc = 0.f;
    const float ri = s_ri[rr];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float wh = w[e] * (ri * s_ci[lane * 8 + e]) - lrr * u[e];
      const float q = wh * wh;
      racc += q;
      colacc[e] += q;
      facc += q;
    }
    if (a.norm_axis == 1 && row < m) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) racc += __shfl_xor_sync(0xffffffffu, racc, o);
      if (lane == 0) part.r[(l * m + row) * gridDim.x + blockIdx.x] = racc;
    }
  }
  if (a.norm_axis == 2) {
#pragma unroll
    for (int e = 0; e < 8; ++e) s_col[warp][lane * 8 + e] = colacc[e];
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < THREADS / 32; ++w) t += s_col[w][threadIdx.x];
    if (c0 + threadIdx.x < n) part.c[(l * gridDim.y + blockIdx.y) * n + c0 + threadIdx.x] = t;
  } else if (a.norm_axis == 0) {
    const float t = block_sum(facc, sh);
    if (threadIdx.x == 0) part.s[l * gridDim.y * gridDim.x + blockIdx.y * gridDim.x + blockIdx.x] = t;
  }
}

struct GainArgs {
  float* raw[3];          // scalar [L], row [L, m], col [L, n] (in/out), null when absent
  float* m1[3];
  float* m2[3];
  const float* red[3];    // reductions from md_pre_kernel
  float* sp_old[3];       // out: softplus of the old / new raw gains
  float* sp_new[3];
  int64_t len[3];
  const float* step_dev;  // gain step after the increment (device) or null
  float step_host;
  float b1, b2, eps, gain_lr;
  const float* ss;        // sums of squares [n_proj]
  const float* target;    // target norms [n_proj]
  float* proj;            // out: target / (sqrt(ss) + 1e-12)
  int64_t n_proj;
};

// Adam on the raw gains with dL/draw = reduction * sigmoid(raw) (all from the old gains),
// raw -= gain_lr * update; and the sphere projection factors.
__global__ void md_gain_kernel(GainArgs a) {
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const float step = a.step_dev != nullptr ? __ldg(a.step_dev) : a.step_host;
  const float bc1 = 1.f - powf(a.b1, step), bc2 = 1.f - powf(a.b2, step);
  for (int k = 0; k < 3; ++k) {
    if (a.raw[k] == nullptr) continue;
    for (int64_t i = tid; i < a.len[k]; i += stride) {
      const float raw = a.raw[k][i];
      const float gr = a.red[k][i] * sigmoid_f(raw);
      const float m1 = lerp_f(a.m1[k][i], gr, 1.f - a.b1);
      const float m2 = lerp_f(a.m2[k][i], gr * gr, 1.f - a.b2);
      a.m1[k][i] = m1;
      a.m2[k][i] = m2;
      const float upd = (m1 / bc1) / (sqrtf(m2 / bc2) + a.eps);
      const float nr = raw + (-a.gain_lr) * upd;
      a.raw[k][i] = nr;
      a.sp_old[k][i] = softplus_f(raw);
      a.sp_new[k][i] = softplus_f(nr);
    }
  }
  for (int64_t i = tid; i < a.n_proj; i += stride) a.proj[i] = a.target[i] / (sqrtf(a.ss[i]) + 1e-12f);
}

struct WriteArgs {
  const float* sp_old[3];  // null when the gain is absent
  const float* sp_new[3];
  const float* proj;
  __nv_bfloat16* shadow;   // nullable: a bf16 copy of the new weights in p's layout (f32 p only)
};

template <bool VEC, bool TRANS, typename TP>
__global__ void __launch_bounds__(THREADS, 2) md_write_kernel(PostArgs a, WriteArgs wa, TP* __restrict__ p) {
  // s_roi / s_coi: reciprocal old gains (row factor with the scalar folded in);
  // s_rf / s_cf: new gains times the projection factor of the tile's rows / columns
  __shared__ float s_roi[TR], s_rf[TR], s_coi[TC], s_cf[TC];
  __shared__ uint32_t s_t[TRANS ? TC : 1][TW];
  extern __shared__ __align__(16) uint8_t md_dyn[];
  uint4* st = reinterpret_cast<uint4*>(md_dyn);
  const int64_t m = a.m, n = a.n;
  const int64_t l = blockIdx.z, r0 = (int64_t)blockIdx.y * TR, c0 = (int64_t)blockIdx.x * TC;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t c = c0 + lane * 8;
  // p may be W itself (the f32 parameter updated in place): every read of W is staged
  // (or, unvectorised, loaded into registers) before the thread's first store
  if constexpr (VEC) stage_rows<TRANS>(st, a.W, a.U, l, m, n, r0, c);
  const float so = wa.sp_old[0] != nullptr ? wa.sp_old[0][l] : 1.f;
  const float sn = wa.sp_new[0] != nullptr ? wa.sp_new[0][l] : 1.f;
  const float pf = a.norm_axis == 0 ? wa.proj[l] : 1.f;
  for (int i = threadIdx.x; i < TR; i += THREADS) {
    const bool ok = wa.sp_old[1] != nullptr && r0 + i < m;
    const float ro = ok ? wa.sp_old[1][l * m + r0 + i] : 1.f;
    const float rn = ok ? wa.sp_new[1][l * m + r0 + i] : 1.f;
    const float pr = a.norm_axis == 1 ? (r0 + i < m ? wa.proj[l * m + r0 + i] : 1.f) : pf;
    s_roi[i] = 1.0f / (so * ro);
    s_rf[i] = (sn * rn) * pr;
  }
  for (int i = threadIdx.x; i < TC; i += THREADS) {
    const bool ok = wa.sp_old[2] != nullptr && c0 + i < n;
    const float co = ok ? wa.sp_old[2][l * n + c0 + i] : 1.f;
    const float cn = ok ? wa.sp_new[2][l * n + c0 + i] : 1.f;
    const float pc = a.norm_axis == 2 && c0 + i < n ? wa.proj[l * n + c0 + i] : 1.f;
    s_coi[i] = 1.0f / co;
    s_cf[i] = cn * pc;
  }
  if constexpr (TRANS) stage_t_load(s_t, a.U, l, m, n, r0, c0, a.u_words);
  if constexpr (VEC || TRANS) cp_async_wait_all();
  __syncthreads();
  const float lrr = lr_of(a) * a.rescale;
  if (c >= n) return;
  float wr[VEC ? 1 : 8][8];
  uint32_t urr[VEC ? 1 : 8][4];
  if constexpr (!VEC) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int64_t row = r0 + warp * 8 + k;
      if (row < m) {
        load8<VEC>(a.W + (l * m + row) * n, c, n, wr[k]);
        if constexpr (!TRANS) load8_bf16_raw<VEC>(a.U + (l * m + row) * n, c, n, urr[k]);
      }
    }
  }
#pragma unroll 2
  for (int k = 0; k < 8; ++k) {
    const int rr = warp * 8 + k;
    const int64_t row = r0 + rr;
    if (row >= m) break;
    const int64_t off = (l * m + row) * n;
    float w[8], u[8], o[8];
    uint32_t ur[4];
    if constexpr (VEC) {
      staged_w(st, k, Stage<TRANS>::NCH, w);
      if constexpr (!TRANS) {
        const uint4 q4 = st[(k * 3 + 2) * THREADS + threadIdx.x];
        ur[0] = q4.x; ur[1] = q4.y; ur[2] = q4.z; ur[3] = q4.w;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) w[e] = wr[k][e];
      if constexpr (!TRANS) {
#pragma unroll
        for (int e = 0; e < 4; ++e) ur[e] = urr[k][e];
      }
    }
    if constexpr (TRANS) stage_t_row(s_t, rr, lane, ur);
    unpack8_bf16(ur, u);
    const float roi = s_roi[rr], rf = s_rf[rr];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      // new gain * projected (W / old gain - lr * rescale * U)
      const float wh = w[e] * (roi * s_coi[lane * 8 + e]) - lrr * u[e];
      o[e] = wh * (rf * s_cf[lane * 8 + e]);
    }
    if constexpr (std::is_same<TP, float>::value) {
      store8<VEC>(p + off, c, n, o);
      if (wa.shadow != nullptr) store8_bf16<VEC>(wa.shadow + off, c, n, o);
    } else {
      store8_bf16<VEC>(p + off, c, n, o);
    }
  }
}

}  // namespace md
}  // namespace zs

using namespace zs;

static bool md_vec_ok(int64_t n, std::initializer_list<const void*> ptrs) {
  if (n % 8 != 0) return false;
  for (const void* p : ptrs)
    if (p != nullptr && (reinterpret_cast<uintptr_t>(p) % 16) != 0) return false;
  return true;
}

static dim3 md_grid(int64_t L, int64_t m, int64_t n) {
  return dim3((unsigned)((n + md::TC - 1) / md::TC), (unsigned)((m + md::TR - 1) / md::TR), (unsigned)L);
}

// floats of the three partial-sum arrays of one pass over [L, m, n]
static int64_t md_partial_floats(int64_t L, int64_t m, int64_t n) {
  const int64_t gx = (n + md::TC - 1) / md::TC, gy = (m + md::TR - 1) / md::TR;
  return L * m * gx + L * gy * n + L * gy * gx;
}

static md::Partials md_partials(float* base, int64_t L, int64_t m, int64_t n) {
  const int64_t gx = (n + md::TC - 1) / md::TC, gy = (m + md::TR - 1) / md::TR;
  return md::Partials{base, base + L * m * gx, base + L * m * gx + L * gy * n};
}

// reduce the partials of one axis into out (0: whole matrix [L], 1: rows [L, m], 2: columns [L, n])
static int md_finish(const md::Partials& p, int axis, float* out, int64_t L, int64_t m, int64_t n,
                     cudaStream_t stream) {
  const int64_t gx = (n + md::TC - 1) / md::TC, gy = (m + md::TR - 1) / md::TR;
  const float* part = axis == 0 ? p.s : (axis == 1 ? p.r : p.c);
  const int64_t count = axis == 0 ? L : (axis == 1 ? L * m : L * n);
  const int64_t inner = axis == 2 ? n : 1;
  const int K = (int)(axis == 0 ? gy * gx : (axis == 1 ? gx : gy));
  int64_t blocks = (count + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  md::md_finish_kernel<<<(unsigned)blocks, 256, 0, stream>>>(part, out, count, inner, K);
  ZS_CUDA_TRY(cudaGetLastError());
  return ZS_OK;
}

extern "C" size_t zs_muonmd_pre_workspace(int64_t L, int64_t m, int64_t n) {
  return (size_t)md_partial_floats(L, m, n) * sizeof(float) + 256;
}

extern "C" int zs_muonmd_pre(const float* W, const float* G, float* buf, const float* g_scalar, const float* g_row,
                             const float* g_col, void* x_out, int x_transposed, float* red_scalar, float* red_row,
                             float* red_col,
                             int64_t L, int64_t m, int64_t n, float momentum, void* workspace,
                             size_t workspace_bytes, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ZS_REQUIRE(W && G && buf && x_out, ZS_ERR_ARG);
  ZS_REQUIRE(L >= 1 && m >= 1 && n >= 1 && L < 65536 && (m + md::TR - 1) / md::TR < 65536, ZS_ERR_SHAPE);
  ZS_REQUIRE((g_scalar == nullptr) == (red_scalar == nullptr) && (g_row == nullptr) == (red_row == nullptr) &&
                 (g_col == nullptr) == (red_col == nullptr),
             ZS_ERR_ARG);
  const bool any_red = red_scalar != nullptr || red_row != nullptr || red_col != nullptr;
  ZS_REQUIRE(!any_red || (workspace && workspace_bytes >= zs_muonmd_pre_workspace(L, m, n)), ZS_ERR_WORKSPACE);
  ZS_BIND(W);
  md::Gains g{g_scalar, g_row, g_col};
  auto* X = reinterpret_cast<__nv_bfloat16*>(x_out);
  const dim3 grid = md_grid(L, m, n);
  float* ws = any_red ? reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255))
                      : nullptr;
  const md::Partials part = any_red ? md_partials(ws, L, m, n) : md::Partials{nullptr, nullptr, nullptr};
  const bool ws_ = red_scalar != nullptr, wr = red_row != nullptr, wc = red_col != nullptr;
  const bool words = m % 2 == 0 && (reinterpret_cast<uintptr_t>(x_out) & 3) == 0;
  const bool vec = x_transposed ? md_vec_ok(n, {W, G, buf}) : md_vec_ok(n, {W, G, buf, x_out});
  auto launch = [&](auto kern) {
    kern<<<grid, md::THREADS, 0, stream>>>(W, G, buf, g, X, part, ws_, wr, wc, m, n, momentum, words);
  };
  if (x_transposed) {
    if (vec) launch(md::md_pre_kernel<true, true>); else launch(md::md_pre_kernel<false, true>);
  } else {
    if (vec) launch(md::md_pre_kernel<true, false>); else launch(md::md_pre_kernel<false, false>);
  }
  ZS_CUDA_TRY(cudaGetLastError());
  int rc;
  if (ws_ && (rc = md_finish(part, 0, red_scalar, L, m, n, stream)) != ZS_OK) return rc;
  if (wr && (rc = md_finish(part, 1, red_row, L, m, n, stream)) != ZS_OK) return rc;
  if (wc && (rc = md_finish(part, 2, red_col, L, m, n, stream)) != ZS_OK) return rc;
  return ZS_OK;
}

extern "C" size_t zs_muonmd_post_workspace(int64_t L, int64_t m, int64_t n) {
  // ss + proj (up to L*max(m,n) each) + softplus old/new of scalar, row, column gains
  // + the reduction pass's partial sums
  const int64_t mx = m > n ? m : n;
  return (size_t)(2 * L * mx + 2 * (L + L * m + L * n) + md_partial_floats(L, m, n)) * sizeof(float) + 8 * 256;
}

extern "C" int zs_muonmd_post(const float* W, const void* U, int u_transposed, void* p_out, int p_dtype,
                              void* shadow_bf16, float* g_scalar, float* g_row,
                              float* g_col, float* m1_scalar, float* m2_scalar, float* m1_row, float* m2_row,
                              float* m1_col, float* m2_col, const float* red_scalar, const float* red_row,
                              const float* red_col, const float* step_dev, float step_host, float b1, float b2,
                              float eps, float gain_lr, const float* lr_dev, float lr_host, float rescale,
                              int norm_axis, const float* target_norm, int64_t L, int64_t m, int64_t n,
                              void* workspace, size_t workspace_bytes, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ZS_REQUIRE(W && U && p_out && target_norm, ZS_ERR_ARG);
  ZS_REQUIRE(p_dtype == ZS_F32 || p_dtype == ZS_BF16, ZS_ERR_DTYPE);
  ZS_REQUIRE(shadow_bf16 == nullptr || p_dtype == ZS_F32, ZS_ERR_ARG);
  ZS_REQUIRE(norm_axis >= 0 && norm_axis <= 2, ZS_ERR_ARG);
  ZS_REQUIRE(L >= 1 && m >= 1 && n >= 1 && L < 65536 && (m + md::TR - 1) / md::TR < 65536, ZS_ERR_SHAPE);
  ZS_REQUIRE((g_scalar == nullptr || (m1_scalar && m2_scalar && red_scalar)) &&
                 (g_row == nullptr || (m1_row && m2_row && red_row)) &&
                 (g_col == nullptr || (m1_col && m2_col && red_col)),
             ZS_ERR_ARG);
  ZS_REQUIRE(workspace && workspace_bytes >= zs_muonmd_post_workspace(L, m, n), ZS_ERR_WORKSPACE);
  ZS_BIND(W);
  const int64_t n_proj = norm_axis == 0 ? L : (norm_axis == 1 ? L * m : L * n);
  float* ws = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  const int64_t mx = m > n ? m : n;
  float* ss = ws;
  float* proj = ss + L * mx;
  float* sp = proj + L * mx;  // old: sc [L], row [L*m], col [L*n]; then new
  float* sp_old[3] = {sp, sp + L, sp + L + L * m};
  float* sp_new[3] = {sp_old[2] + L * n, sp_old[2] + L * n + L, sp_old[2] + L * n + L + L * m};
  const md::Partials part = md_partials(sp_new[2] + L * n, L, m, n);
  md::PostArgs a{W, reinterpret_cast<const __nv_bfloat16*>(U), m, n, lr_dev, lr_host, rescale, norm_axis,
                 m % 2 == 0 && (reinterpret_cast<uintptr_t>(U) & 3) == 0};
  md::Gains g{g_scalar, g_row, g_col};
  const dim3 grid = md_grid(L, m, n);
  const bool vec = u_transposed ? md_vec_ok(n, {W, p_out, shadow_bf16}) : md_vec_ok(n, {W, U, p_out, shadow_bf16});
  // the vectorised passes stage their rows in dynamic shared memory (md::Stage)
  auto reduce = [&](auto kern, int dyn) -> int {
    if (dyn > 0) ZS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn));
    kern<<<grid, md::THREADS, dyn, stream>>>(a, g, part);
    return ZS_OK;
  };
  int rc0;
  if (u_transposed)
    rc0 = vec ? reduce(md::md_reduce_kernel<true, true>, md::Stage<true>::BYTES)
              : reduce(md::md_reduce_kernel<false, true>, 0);
  else
    rc0 = vec ? reduce(md::md_reduce_kernel<true, false>, md::Stage<false>::BYTES)
              : reduce(md::md_reduce_kernel<false, false>, 0);
  if (rc0 != ZS_OK) return rc0;
  ZS_CUDA_TRY(cudaGetLastError());
  {
    const int rc = md_finish(part, norm_axis, ss, L, m, n, stream);
    if (rc != ZS_OK) return rc;
  }
  md::GainArgs ga{};
  float* raws[3] = {g_scalar, g_row, g_col};
  float* m1s[3] = {m1_scalar, m1_row, m1_col};
  float* m2s[3] = {m2_scalar, m2_row, m2_col};
  const float* reds[3] = {red_scalar, red_row, red_col};
  const int64_t lens[3] = {L, L * m, L * n};
  md::WriteArgs wa{};
  for (int k = 0; k < 3; ++k) {
    ga.raw[k] = raws[k];
    ga.m1[k] = m1s[k];
    ga.m2[k] = m2s[k];
    ga.red[k] = reds[k];
    ga.sp_old[k] = sp_old[k];
    ga.sp_new[k] = sp_new[k];
    ga.len[k] = lens[k];
    wa.sp_old[k] = raws[k] != nullptr ? sp_old[k] : nullptr;
    wa.sp_new[k] = raws[k] != nullptr ? sp_new[k] : nullptr;
  }
  ga.step_dev = step_dev;
  ga.step_host = step_host;
  ga.b1 = b1;
  ga.b2 = b2;
  ga.eps = eps;
  ga.gain_lr = gain_lr;
  ga.ss = ss;
  ga.target = target_norm;
  ga.proj = proj;
  ga.n_proj = n_proj;
  wa.proj = proj;
  wa.shadow = reinterpret_cast<__nv_bfloat16*>(shadow_bf16);
  const int64_t work = n_proj > L * (1 + m + n) ? n_proj : L * (1 + m + n);
  int64_t blocks = (work + 255) / 256;
  if (blocks > 148 * 4) blocks = 148 * 4;
  md::md_gain_kernel<<<(unsigned)blocks, 256, 0, stream>>>(ga);
  ZS_CUDA_TRY(cudaGetLastError());
  auto launch_write = [&](auto kern, int dyn, auto* out_typed) -> int {
    if (dyn > 0) ZS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn));
    kern<<<grid, md::THREADS, dyn, stream>>>(a, wa, out_typed);
    return ZS_OK;
  };
  auto write = [&](auto* out_typed) -> int {
    using TP = std::remove_pointer_t<decltype(out_typed)>;
    if (u_transposed)
      return vec ? launch_write(md::md_write_kernel<true, true, TP>, md::Stage<true>::BYTES, out_typed)
                 : launch_write(md::md_write_kernel<false, true, TP>, 0, out_typed);
    return vec ? launch_write(md::md_write_kernel<true, false, TP>, md::Stage<false>::BYTES, out_typed)
               : launch_write(md::md_write_kernel<false, false, TP>, 0, out_typed);
  };
  const int rc1 = p_dtype == ZS_F32 ? write(reinterpret_cast<float*>(p_out))
                                    : write(reinterpret_cast<__nv_bfloat16*>(p_out));
  if (rc1 != ZS_OK) return rc1;
  ZS_CUDA_TRY(cudaGetLastError());
  return ZS_OK;
}
