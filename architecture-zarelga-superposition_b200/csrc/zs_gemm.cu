// Grouped expert GEMMs on the 5th-generation tensor cores (tcgen05 + TMEM),
// fed by TMA.  One persistent, warp-specialised kernel template covers every
// contraction of the scattermoe expert layer:
//
//   MODE_ROWS  out[rows of expert e, :] = A[rows, :K] @ B_e^T
//              (scatter2scatter, scattermoe/kernels/ops.py:128-190; forward
//               up/down projections and the input-gradient GEMMs)
//   MODE_XTY   out_e = A[rows of e]^T @ B[rows of e]
//              (groupXtY, scattermoe/kernels/ops.py:320-438; weight gradients)
//
// Warp roles (320 threads, one CTA per SM):
//   warp 0      TMA producer (one elected lane) + TMEM allocator
//   warp 1      MMA issuer (lane 0 issues tcgen05.mma, whole warp zero-fills
//               reduction tails in MODE_XTY)
//   warps 2..9  epilogue: tcgen05.ld TMEM -> registers -> per-warp shared
//               memory transpose -> 64-byte row-segment global stores
// Pipelines: STAGES shared-memory stages (full/empty mbarriers) between the
// producer and the MMA warp; two TMEM accumulator buffers (tfull/tempty)
// between the MMA warp and the epilogue, so the epilogue of tile i overlaps
// the main loop of tile i+1.
//
// Tiles are 128 x BN x 64 (BM x BN x BK), bf16/f16 operands in 128-byte
// swizzled shared memory, f32 accumulation in TMEM.  A tile never spans two
// experts: every expert's rows start a new M tile, and the tile list is built
// on the device from the expert boundaries, so no host sync is needed.
#include "zs_common.cuh"

#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>

namespace zs {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int MAX_EXPERTS_GEMM = 1024;

enum { MODE_ROWS = 0, MODE_XTY = 1 };
enum { EPI_STORE = 0, EPI_SWIGLU = 1, EPI_DSWIGLU = 2, EPI_LSE = 3, EPI_XENT_GRAD = 4, EPI_F32 = 5, EPI_AXPBY = 6 };

struct GemmArgs {
  int mode;
  int num_experts;
  int n_tiles;           // output tiles along N
  int m_tiles_xty;       // MODE_XTY: tiles along M
  int kb_rows;           // MODE_ROWS: number of BK blocks along K
  int M_xty;             // MODE_XTY: M extent (masking)
  int N_out;             // output columns (masking)
  int ab_fmt;            // 0 = f16, 1 = bf16
  int64_t n_rows;        // sorted rows in total
  int64_t out_rows;      // MODE_ROWS: rows of the output (row_map values must lie below)
  const int64_t* expert_offsets;      // inclusive cumsum, or null
  const int64_t* sorted_expert_idxs;  // used when expert_offsets is null
  const int64_t* row_map;             // MODE_ROWS: output row per sorted row (null: identity)
  char* out;
  int64_t ldo_m, ldo_n, out_se;       // element strides of the output
  char* out2;                          // EPI_SWIGLU: pre-activation rows (nullable)
  int64_t ldo2;
  const char* bias;                    // MODE_ROWS + EPI_STORE (nullable)
  int64_t bias_se, bias_sn;
  int out_dtype;                       // ZS_F32 / ZS_BF16 / ZS_F16
  int b_rows_per_expert;               // rows of B's 2-D view per expert
  int swiglu_half;                     // EPI_SWIGLU: B-row offset of the gate half; EPI_DSWIGLU: column
                                       // offset of the gate half in aux/out
  const char* aux;                     // EPI_DSWIGLU: saved pre-activation rows [h | g]
  int64_t ld_aux;
  int vec_ok;                          // 16-byte vector stores allowed for row-contiguous output
  int64_t b_row_offset;                // added to B's row coordinate (dense GEMMs over a slice of B)
  // cross-entropy epilogues (EPI_LSE, EPI_XENT_GRAD); columns are vocabulary entries
  const int64_t* labels;               // [rows, s_max]
  const int* s_count;                  // [rows] active labels per row (0 = row ignored)
  int s_max;
  int64_t col_offset;                  // vocabulary index of this launch's column 0
  float* part_max;                     // EPI_LSE: [rows, part_ld] running max / sum partials
  float* part_sum;
  int64_t part_ld;
  float* target_sum;                   // EPI_LSE: [rows] += target logits (atomic)
  const float* lse;                    // EPI_XENT_GRAD: [rows]
  const float* grad_loss;              // EPI_XENT_GRAD: device scalar dL/dloss
  const float* denom;                  // EPI_XENT_GRAD: device scalar N (total active labels)
  int accumulate;                      // EPI_F32: out += acc instead of out = acc
  const float* f32_scale;              // EPI_F32 (nullable): device scalar multiplying the accumulator
  int64_t group_rows;                  // > 0: uniform groups (batched GEMM), group e = rows [e*g, (e+1)*g)
  float alpha, beta;                   // EPI_AXPBY: out = alpha * acc + beta * aux
  int sym_upper;                       // uniform square groups (pair tiles): the product is symmetric,
                                       // only tiles (i, j >= i) are computed, strictly-upper ones also
                                       // write their transpose (EPI_STORE / EPI_AXPBY)
  int tma_store;                       // EPI_STORE / EPI_AXPBY without row_map or bias: full 32 x 32
                                       // chunks go out through the third tensor map (TMA stores)
  int sym_ops;                         // uniform square groups on pair tiles: bit 0 (A), bit 1 (B): the
                                       // operand is a symmetric matrix of which only the upper 256 x 256
                                       // tiles are stored; a k-block left of the diagonal tile is read
                                       // transposed (MN-major) from tmAT / tmBT.  With sym_ops the
                                       // symmetric products' outputs skip their mirrored lower tiles.
};

template <int BN, int STAGES, bool PAIR = false>
struct Smem {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = (PAIR ? BN / 2 : BN) * BK * 2;   // a CTA pair splits B along N
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int OFF_STAGES = 0;
  static constexpr int OFF_BARS = STAGES * STAGE_BYTES;
  // full[S], empty[S], tfull[2], tempty[2], done
  static constexpr int NUM_BARS = 2 * STAGES + 5;
  static constexpr int OFF_MISC = OFF_BARS + NUM_BARS * 8;  // tmem addr, abort flag
  static constexpr int OFF_TPREFIX = OFF_MISC + 16;
  static constexpr int OFF_RSTART = OFF_TPREFIX + (MAX_EXPERTS_GEMM + 1) * 4;
  static constexpr int OFF_ORDER = OFF_RSTART + (MAX_EXPERTS_GEMM + 1) * 4;
  // per-warp staging buffers start on 512-byte boundaries (the TMA-store box's swizzle atom)
  static constexpr int OFF_STG = ((OFF_ORDER + (MAX_EXPERTS_GEMM + 1) * 4 + 1023) / 1024) * 1024;
  static constexpr int TOTAL = OFF_STG + 8 * 32 * 80;
  static constexpr int ALLOC = TOTAL + 1024;  // slack for 1024-byte alignment
};

struct TileInfo {
  int e;
  int mt, nt;
  int r0, r1;   // MODE_ROWS: rows [r0, r1) of this tile; MODE_XTY: expert rows [r0, r1)
  int nkb;      // k-blocks in the main loop
};

__device__ __forceinline__ int64_t lower_bound_i64(const int64_t* a, int64_t n, int64_t v) {
  int64_t lo = 0, hi = n;
  while (lo < hi) {
    int64_t mid = (lo + hi) >> 1;
    if (__ldg(a + mid) < v)
      lo = mid + 1;
    else
      hi = mid;
  }
  return lo;
}

// Tiles are numbered expert by expert in the order order[0..E); tprefix[p] is
// the first tile of the expert at position p.
template <int BN, int TM>
__device__ __forceinline__ TileInfo decode_tile(int t, const GemmArgs& a, const int* tprefix, const int* rstart,
                                                const int* order) {
  TileInfo ti;
  int lo = 0, hi = a.num_experts;
  while (hi - lo > 1) {
    int mid = (lo + hi) >> 1;
    if (tprefix[mid] <= t)
      lo = mid;
    else
      hi = mid;
  }
  int local = t - tprefix[lo];
  lo = order[lo];
  ti.e = lo;
  if (a.sym_upper) {
    // row i holds tiles (i, i..n_tiles-1)
    int i = 0;
    while (local >= a.n_tiles - i) {
      local -= a.n_tiles - i;
      ++i;
    }
    ti.mt = i;
    ti.nt = i + local;
  } else {
    // Row tiles of a group whose output is wider than it is tall (N > rows, e.g. the
    // classifier GEMM of the cut cross entropy) go column by column: the CTAs in flight
    // then share a few column tiles of B and revisit the (smaller) A from L2, so B
    // streams from DRAM once instead of once per row tile.  Otherwise row by row.
    const int rows_g = rstart[lo + 1] - rstart[lo];
    const int n_mt = (rows_g + TM - 1) / TM;
    if (a.mode == MODE_ROWS && n_mt > 1 && (int64_t)a.n_tiles * BN > (int64_t)rows_g) {
      ti.nt = local / n_mt;
      ti.mt = local - ti.nt * n_mt;
    } else {
      ti.mt = local / a.n_tiles;
      ti.nt = local - ti.mt * a.n_tiles;
    }
  }
  if (a.mode == MODE_ROWS) {
    ti.r0 = rstart[lo] + ti.mt * TM;
    ti.r1 = min(ti.r0 + TM, rstart[lo + 1]);
    ti.nkb = a.kb_rows;
  } else {
    ti.r0 = rstart[lo];
    ti.r1 = rstart[lo + 1];
    ti.nkb = (ti.r1 - ti.r0 + BK - 1) / BK;
  }
  return ti;
}

__device__ __forceinline__ void store_val(char* base, int64_t idx, int dtype, float v) {
  if (dtype == ZS_BF16)
    reinterpret_cast<__nv_bfloat16*>(base)[idx] = __float2bfloat16_rn(v);
  else if (dtype == ZS_F16)
    reinterpret_cast<__half*>(base)[idx] = __float2half_rn(v);
  else
    reinterpret_cast<float*>(base)[idx] = v;
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi, int dtype) {
  if (dtype == ZS_F16) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&b);
}

__device__ __forceinline__ float round_to(float v, int dtype) {
  if (dtype == ZS_BF16) return __bfloat162float(__float2bfloat16_rn(v));
  if (dtype == ZS_F16) return __half2float(__float2half_rn(v));
  return v;
}

// Fast sigmoid / silu in f32 (ex2.approx-based exp and approximate divide);
// the result is rounded to the storage dtype by the caller, which hides the
// few-ulp f32 difference from torch's x / (1 + exp(-x)).
__device__ __forceinline__ float sigmoid_fast(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }
__device__ __forceinline__ float silu_fast(float x) { return x * sigmoid_fast(x); }

// Per-warp staging buffer for coalesced row stores: 32 rows x 64 bytes with
// an 80-byte pitch (conflict-free 16-byte writes and reads).
constexpr int STG_PITCH = 80;
constexpr int STG_BYTES = 32 * STG_PITCH;
constexpr int NUM_EPI_WARPS = 8;

// Write 32 consecutive 16-bit columns [col0, col0 + ncols) of this lane's
// output row (element (row, n) at out[row_off + n]), given as 16 packed pairs.
// When the chunk is full and aligned, the warp transposes its 32 rows through
// shared memory so that each store instruction writes 64 contiguous bytes of
// 8 rows; otherwise scalar stores.  Must be called by all 32 lanes with
// warp-uniform col0/ncols.
template <int DT>
__device__ __forceinline__ void emit_packed(char* out, int64_t row_off, int col0, int ncols, bool valid,
                                            const uint32_t (&p)[16], bool vec, uint8_t* stg) {
  const int lane = threadIdx.x & 31;
  if (vec && ncols == 32) {
    uint4* my = reinterpret_cast<uint4*>(stg + lane * STG_PITCH);
#pragma unroll
    for (int q = 0; q < 4; ++q) my[q] = make_uint4(p[4 * q], p[4 * q + 1], p[4 * q + 2], p[4 * q + 3]);
    __syncwarp();
    const unsigned long long my_ptr =
        valid ? reinterpret_cast<unsigned long long>(out + (row_off + col0) * 2) : 0ull;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = 8 * i + (lane >> 2);
      const int qq = lane & 3;
      const uint4 w = *reinterpret_cast<const uint4*>(stg + r * STG_PITCH + qq * 16);
      const unsigned long long ptr = __shfl_sync(0xffffffffu, my_ptr, r);
      if (ptr != 0ull) reinterpret_cast<uint4*>(ptr)[qq] = w;
    }
    __syncwarp();
  } else if (valid) {
    uint16_t* o = reinterpret_cast<uint16_t*>(out) + row_off + col0;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < ncols) o[j] = (j & 1) ? (uint16_t)(p[j >> 1] >> 16) : (uint16_t)(p[j >> 1] & 0xffffu);
  }
}

template <int DT>
__device__ __forceinline__ void emit_chunk(char* out, int64_t row_off, int col0, int ncols, bool valid,
                                           const float (&v)[32], bool vec, uint8_t* stg) {
  uint32_t p[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) p[j] = pack2(v[2 * j], v[2 * j + 1], DT);
  emit_packed<DT>(out, row_off, col0, ncols, valid, p, vec, stg);
}

// The transpose of a warp's 32 rows x 32 columns chunk: lane l writes output
// row mrow0 + l, columns [mcol0, mcol0 + 32) (64 contiguous bytes), i.e. the
// chunk's column l.  Through the warp's staging buffer.
__device__ __forceinline__ void emit_packed_mirror(char* out, int64_t ldo, int64_t mrow0, int64_t mcol0,
                                                   const uint32_t (&p)[16], uint8_t* stg) {
  const int lane = threadIdx.x & 31;
  uint4* my = reinterpret_cast<uint4*>(stg + lane * STG_PITCH);
#pragma unroll
  for (int q = 0; q < 4; ++q) my[q] = make_uint4(p[4 * q], p[4 * q + 1], p[4 * q + 2], p[4 * q + 3]);
  __syncwarp();
  uint32_t t[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint32_t lo = *reinterpret_cast<const uint16_t*>(stg + (2 * i) * STG_PITCH + lane * 2);
    const uint32_t hi = *reinterpret_cast<const uint16_t*>(stg + (2 * i + 1) * STG_PITCH + lane * 2);
    t[i] = lo | (hi << 16);
  }
  __syncwarp();
  uint4* dst = reinterpret_cast<uint4*>(out + ((mrow0 + lane) * ldo + mcol0) * 2);
#pragma unroll
  for (int q = 0; q < 4; ++q) dst[q] = make_uint4(t[4 * q], t[4 * q + 1], t[4 * q + 2], t[4 * q + 3]);
}

// One warp's 32 x 32 chunk of 16-bit outputs (lane = row, 16 packed pairs)
// through its staging buffer to global memory by a TMA store at column c0,
// row r0 of tmO (box 32 x 32, 64-byte swizzle: 16-byte unit u of buffer row j
// sits at unit u ^ ((j >> 1) & 3)).  transposed: the chunk's column j becomes
// buffer row j (the mirror of a symmetric tile).  The buffer is reused only
// after the previous store from it has been read.
__device__ __forceinline__ void tma_emit_chunk(const CUtensorMap* tmO, uint8_t* stg, const uint32_t (&p)[16], int c0,
                                               int r0, bool transposed) {
  const int lane = threadIdx.x & 31;
  if (lane == 0) bulk_wait_read_all();
  __syncwarp();
  if (!transposed) {
    const int sw = (lane >> 1) & 3;
#pragma unroll
    for (int q = 0; q < 4; ++q)
      *reinterpret_cast<uint4*>(stg + lane * 64 + ((q ^ sw) << 4)) =
          make_uint4(p[4 * q], p[4 * q + 1], p[4 * q + 2], p[4 * q + 3]);
  } else {
    // value 2i of this lane -> (row 2i, column lane), value 2i+1 -> (row 2i+1, column lane)
    const int u = lane >> 3, b = (lane & 7) * 2;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int off = ((u ^ (i & 3)) << 4) + b;
      *reinterpret_cast<uint16_t*>(stg + (2 * i) * 64 + off) = (uint16_t)(p[i] & 0xffffu);
      *reinterpret_cast<uint16_t*>(stg + (2 * i + 1) * 64 + off) = (uint16_t)(p[i] >> 16);
    }
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(tmO, stg, c0, r0);
    bulk_commit();
  }
}

// Read 32 consecutive 16-bit columns of this lane's row as f32.
__device__ __forceinline__ void load_chunk(const char* src, int64_t row_off, int col0, int ncols, bool valid,
                                           float (&v)[32], int dtype, bool vec) {
  if (!valid) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = 0.f;
    return;
  }
  if (vec && ncols == 32) {
    const uint4* p = reinterpret_cast<const uint4*>(src + (row_off + col0) * 2);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 w = __ldg(p + q);
      const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        if (dtype == ZS_F16) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u[h]));
          v[q * 8 + 2 * h] = f.x;
          v[q * 8 + 2 * h + 1] = f.y;
        } else {
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u[h]));
          v[q * 8 + 2 * h] = f.x;
          v[q * 8 + 2 * h + 1] = f.y;
        }
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      float x = 0.f;
      if (j < ncols) {
        const int64_t i = row_off + col0 + j;
        if (dtype == ZS_BF16)
          x = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(src)[i]);
        else
          x = __half2float(reinterpret_cast<const __half*>(src)[i]);
      }
      v[j] = x;
    }
  }
}

// Two 16-bit lanes of a packed word <-> f32 pair; and the product of two
// packed pairs rounded once to the 16-bit type (exact f32 product of two
// 16-bit values, then round-to-nearest: the reference's `a * b` on tensors).
template <int DT>
__device__ __forceinline__ float2 unpk(uint32_t u) {
  if (DT == ZS_F16) return __half22float2(*reinterpret_cast<const __half2*>(&u));
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
}
template <int DT>
__device__ __forceinline__ uint32_t pk(float a, float b) {
  return pack2(a, b, DT);
}
template <int DT>
__device__ __forceinline__ uint32_t mul_rn(uint32_t a, uint32_t b) {
  const float2 x = unpk<DT>(a), y = unpk<DT>(b);
  return pack2(x.x * y.x, x.y * y.y, DT);
}
__device__ __forceinline__ uint32_t word_of(const uint4 (&w)[4], int jj) {
  const uint4& q = w[jj >> 2];
  const int k = jj & 3;
  return k == 0 ? q.x : (k == 1 ? q.y : (k == 2 ? q.z : q.w));
}

// 32 f32 accumulator columns of this lane's row to f32 memory (optionally
// added to what is there).  vec: 16-byte aligned row segments.
__device__ __forceinline__ void store_f32_chunk(float* o, const uint32_t (&r)[32], int ncols, bool acc, bool vec) {
  if (vec && ncols == 32) {
    float4* p = reinterpret_cast<float4*>(o);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float4 v = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]), __uint_as_float(r[4 * q + 2]),
                             __uint_as_float(r[4 * q + 3]));
      if (acc) {
        const float4 w = p[q];
        v.x += w.x;
        v.y += w.y;
        v.z += w.z;
        v.w += w.w;
      }
      p[q] = v;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < ncols) o[j] = (acc ? o[j] : 0.f) + __uint_as_float(r[j]);
  }
}

// The up half [col0, +32) (h) and the gate half [swiglu_half + col0, +32) (g) of
// this lane's saved row, raw.
__device__ __forceinline__ void prefetch_chunk(const GemmArgs& a, int64_t row, int col0, bool ok, uint4 (&h)[4],
                                               uint4 (&g)[4]) {
  ok = ok && col0 + 32 <= a.N_out;
  const uint4* ph = reinterpret_cast<const uint4*>(a.aux + (row * a.ld_aux + col0) * 2);
  const uint4* pg = reinterpret_cast<const uint4*>(a.aux + (row * a.ld_aux + a.swiglu_half + col0) * 2);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    h[q] = ok ? __ldg(ph + q) : make_uint4(0, 0, 0, 0);
    g[q] = ok ? __ldg(pg + q) : make_uint4(0, 0, 0, 0);
  }
}

// PAIR: a cluster of two CTAs computes 256-row MODE_ROWS tiles with one
// tcgen05.mma.cta_group::2 of M = 256 issued by rank 0: each CTA loads its
// 128 rows of A and its half of B's N columns; the stage's bytes of both CTAs
// complete on rank 0's full barrier; rank 0's commits arrive on both CTAs'
// empty / accumulator-full barriers; the epilogue warps of both CTAs release
// the accumulator on rank 0's barrier.
template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI, int DT, bool PAIR>
__global__ void __launch_bounds__(64 + 32 * NUM_EPI_WARPS, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmAT,
                        const __grid_constant__ CUtensorMap tmBT, const GemmArgs args) {
  using L = Smem<BN, STAGES, PAIR>;
  static_assert(!PAIR || !A_MN, "pair tiles are MODE_ROWS only");
  constexpr int TM = PAIR ? 2 * BM : BM;    // rows of a MODE_ROWS tile
  const uint32_t crank = PAIR ? cluster_ctarank() : 0u;
  const int t_first = PAIR ? (int)cluster_id_x() : (int)blockIdx.x;
  const int t_step = PAIR ? (int)cluster_count_x() : (int)gridDim.x;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BARS);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = bars + 2 * STAGES + 2;
  uint64_t* done = bars + 2 * STAGES + 4;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);
  int* s_tprefix = reinterpret_cast<int*>(smem + L::OFF_TPREFIX);
  int* s_rstart = reinterpret_cast<int*>(smem + L::OFF_RSTART);
  int* s_order = reinterpret_cast<int*>(smem + L::OFF_ORDER);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int E = args.num_experts;
  constexpr int TMEM_COLS = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;

  // ---- set-up: barriers, TMEM, expert boundaries
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], NUM_EPI_WARPS * (PAIR ? 2 : 1));   // one arrival per epilogue warp
    }
    mbar_init(done, 1);
    *s_abort = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    if (PAIR) {
      tmem_alloc_pair(s_tmem, TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(s_tmem, TMEM_COLS);
      tmem_relinquish();
    }
  }
  if (warp == 1 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  for (int e = threadIdx.x; e <= E; e += blockDim.x) {
    int64_t s;
    if (e == 0)
      s = 0;
    else if (args.group_rows > 0)
      s = (int64_t)e * args.group_rows;  // batched GEMM with uniform groups
    else if (args.expert_offsets == nullptr && args.sorted_expert_idxs == nullptr)
      s = args.n_rows;  // dense GEMM: one group holding every row
    else if (args.expert_offsets != nullptr)
      s = __ldg(args.expert_offsets + (e - 1));
    else
      s = lower_bound_i64(args.sorted_expert_idxs, args.n_rows, e);
    s = s < 0 ? 0 : (s > args.n_rows ? args.n_rows : s);
    s_rstart[e] = (int)s;
  }
  __syncthreads();
  // Expert order.  MODE_XTY tiles cost in proportion to their expert's rows
  // and the loads are skewed, so the weight-gradient tiles go largest expert
  // first (greedy longest-first over the persistent CTAs); MODE_ROWS tiles
  // all cost the same and keep expert order.
  const bool lpt = args.mode == MODE_XTY && E <= 256;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    if (lpt) {
      const int ce = max(s_rstart[e + 1] - s_rstart[e], 0);
      int rank = 0;
      for (int j = 0; j < E; ++j) {
        const int cj = max(s_rstart[j + 1] - s_rstart[j], 0);
        rank += (cj > ce) || (cj == ce && j < e);
      }
      s_order[rank] = e;
    } else {
      s_order[e] = e;
    }
  }
  __syncthreads();
  if (warp == 0) {
    const int per = (E + 31) / 32;
    const int beg = lane * per;
    const int end = min(beg + per, E);
    int local = 0;
    for (int p = beg; p < end; ++p) {
      const int e = s_order[p];
      int cnt = max(s_rstart[e + 1] - s_rstart[e], 0);
      local += (args.mode == MODE_ROWS) ? (args.sym_upper ? args.n_tiles * (args.n_tiles + 1) / 2
                                                          : ((cnt + TM - 1) / TM) * args.n_tiles)
                                        : args.m_tiles_xty * args.n_tiles;
    }
    int incl = local;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      int v = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += v;
    }
    int run = incl - local;
    for (int p = beg; p < end; ++p) {
      s_tprefix[p] = run;
      const int e = s_order[p];
      int cnt = max(s_rstart[e + 1] - s_rstart[e], 0);
      run += (args.mode == MODE_ROWS) ? (args.sym_upper ? args.n_tiles * (args.n_tiles + 1) / 2
                                                        : ((cnt + TM - 1) / TM) * args.n_tiles)
                                      : args.m_tiles_xty * args.n_tiles;
    }
    if (lane == 31) s_tprefix[E] = incl;
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync_all();   // both CTAs' barriers initialised before any cross-CTA arrival
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;
  const int total_tiles = s_tprefix[E];

  constexpr uint32_t STAGE_TX = (uint32_t)L::STAGE_BYTES;
  constexpr uint32_t IDESC_BF16 = idesc_f16(TM, BN, 1, A_MN ? 1 : 0, B_MN ? 1 : 0);
  constexpr uint32_t IDESC_F16 = idesc_f16(TM, BN, 0, A_MN ? 1 : 0, B_MN ? 1 : 0);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0;       // stages that received at least one load
      uint32_t issued_parity = 0;     // parity of the last load per stage
      bool ok = true;
      for (int t = t_first; t < total_tiles && ok; t += t_step) {
        const TileInfo ti = decode_tile<BN, TM>(t, args, s_tprefix, s_rstart, s_order);
        for (int kb = 0; kb < ti.nkb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, s_abort, ZS_DEVERR_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          uint8_t* sA = smem + L::OFF_STAGES + stage * L::STAGE_BYTES;
          uint8_t* sB = sA + L::A_BYTES;
          if (PAIR) {
            // rank 0's barrier counts both CTAs' bytes; rank 1's loads land
            // in its own shared memory and complete on rank 0's barrier
            if (crank == 0) mbar_arrive_expect_tx(&full[stage], 2 * STAGE_TX);
            if (!B_MN) {
              const int brow = ti.e * args.b_rows_per_expert + (int)args.b_row_offset;
              const int r = EPI == EPI_SWIGLU ? brow + (crank ? args.swiglu_half : 0) + ti.nt * (BN / 2)
                                              : brow + ti.nt * BN + (int)crank * (BN / 2);
              const int kt = (kb * BK) / TM;   // 256-wide tile of this k-block
              if ((args.sym_ops & 1) && kt < ti.mt) {
                // A[rows, k-block] = A[k-block, rows]^T: two 64-column boxes, MN-major
                const int gbase = ti.r0 - ti.mt * TM;
                const int il = ti.mt * TM + (int)crank * BM;
#pragma unroll
                for (int j = 0; j < BM / 64; ++j)
                  tma_load_2d_pair(sA + j * (BK * 128), &tmAT, &full[stage], il + j * 64, gbase + kb * BK);
              } else {
                tma_load_2d_pair(sA, &tmA, &full[stage], kb * BK, ti.r0 + (int)crank * BM);
              }
              if ((args.sym_ops & 2) && kt < ti.nt) {
                const int nl = ti.nt * BN + (int)crank * (BN / 2);
#pragma unroll
                for (int j = 0; j < BN / 128; ++j)
                  tma_load_2d_pair(sB + j * (BK * 128), &tmBT, &full[stage], nl + j * 64, brow + kb * BK);
              } else {
                tma_load_2d_pair(sB, &tmB, &full[stage], kb * BK, r);
              }
            } else {
              const int brow = ti.e * args.b_rows_per_expert + (int)args.b_row_offset + kb * BK;
              if ((args.sym_ops & 1) && (kb * BK) / TM < ti.mt) {
                const int gbase = ti.r0 - ti.mt * TM;
                const int il = ti.mt * TM + (int)crank * BM;
#pragma unroll
                for (int j = 0; j < BM / 64; ++j)
                  tma_load_2d_pair(sA + j * (BK * 128), &tmAT, &full[stage], il + j * 64, gbase + kb * BK);
              } else {
                tma_load_2d_pair(sA, &tmA, &full[stage], kb * BK, ti.r0 + (int)crank * BM);
              }
#pragma unroll
              for (int j = 0; j < BN / 128; ++j)
                tma_load_2d_pair(sB + j * (BK * 128), &tmB, &full[stage], ti.nt * BN + (int)crank * (BN / 2) + j * 64,
                                 brow);
            }
          } else if (args.mode == MODE_ROWS) {
            mbar_arrive_expect_tx(&full[stage], STAGE_TX);
            if (!A_MN) tma_load_2d(sA, &tmA, &full[stage], kb * BK, ti.r0);
            if (!B_MN) {
              // B boxes are 128 rows: two loads per 256-row tile
              const int brow = ti.e * args.b_rows_per_expert + (int)args.b_row_offset;
              if (EPI == EPI_SWIGLU) {
                tma_load_2d(sB, &tmB, &full[stage], kb * BK, brow + ti.nt * (BN / 2));
                tma_load_2d(sB + (BN / 2) * 128, &tmB, &full[stage], kb * BK,
                            brow + args.swiglu_half + ti.nt * (BN / 2));
              } else {
                tma_load_2d(sB, &tmB, &full[stage], kb * BK, brow + ti.nt * BN);
                tma_load_2d(sB + (BN / 2) * 128, &tmB, &full[stage], kb * BK, brow + ti.nt * BN + BN / 2);
              }
            } else {
              const int brow = ti.e * args.b_rows_per_expert + (int)args.b_row_offset + kb * BK;
#pragma unroll
              for (int j = 0; j < BN / 64; ++j)
                tma_load_2d(sB + j * (BK * 128), &tmB, &full[stage], ti.nt * BN + j * 64, brow);
            }
          } else {
            mbar_arrive_expect_tx(&full[stage], STAGE_TX);
            const int row = ti.r0 + kb * BK;
#pragma unroll
            for (int j = 0; j < BM / 64; ++j)
              tma_load_2d(sA + j * (BK * 128), &tmA, &full[stage], ti.mt * BM + j * 64, row);
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(sB + j * (BK * 128), &tmB, &full[stage], ti.nt * BN + j * 64, row);
          }
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Drain: never leave the CTA with a TMA write still in flight.  In a
      // pair, rank 0's full barriers count both CTAs' writes; rank 1 is held
      // by the cluster barrier at the end until rank 0 has drained.
      if (!PAIR || crank == 0)
        for (int s = 0; s < STAGES; ++s)
          if (issued_mask & (1u << s)) mbar_wait(&full[s], (issued_parity >> s) & 1, nullptr, ZS_DEVERR_TIMEOUT_DRAIN);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    int stage = 0;
    uint32_t phase = 0;
    uint32_t acc_iter = 0;
    bool ok = true;
    const uint32_t idesc = DT == ZS_BF16 ? IDESC_BF16 : IDESC_F16;
    bool issued_any = false;
    for (int t = t_first; t < total_tiles && ok && (!PAIR || crank == 0); t += t_step) {
      const TileInfo ti = decode_tile<BN, TM>(t, args, s_tprefix, s_rstart, s_order);
      if (ti.nkb == 0) continue;
      const uint32_t buf = acc_iter & 1;
      const uint32_t acc_phase = (acc_iter >> 1) & 1;
      if (!warp_wait(&tempty[buf], acc_phase ^ 1, s_abort, ZS_DEVERR_TIMEOUT_MMA)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + buf * BN;
      for (int kb = 0; kb < ti.nkb; ++kb) {
        if (!warp_wait(&full[stage], phase, s_abort, ZS_DEVERR_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint8_t* sA = smem + L::OFF_STAGES + stage * L::STAGE_BYTES;
        uint8_t* sB = sA + L::A_BYTES;
        if (args.mode == MODE_XTY) {
          // Reduction tail: rows past the expert's end belong to the next
          // expert.  Zero them in both operands (K-rows of the MN-major tiles).
          const int valid = min(BK, ti.r1 - (ti.r0 + kb * BK));
          if (valid < BK) {
            const int nrow = BK - valid;
            const int chunks_a = (BM / 64) * nrow * 8;
            const int chunks_b = (BN / 64) * nrow * 8;
            const uint4 z = make_uint4(0, 0, 0, 0);
            for (int c = lane; c < chunks_a + chunks_b; c += 32) {
              const bool isA = c < chunks_a;
              const int cc = isA ? c : c - chunks_a;
              const int atom = cc / (nrow * 8);
              const int rem = cc - atom * nrow * 8;
              const int row = valid + (rem >> 3);
              const int ch = rem & 7;
              uint8_t* base = isA ? sA : sB;
              *reinterpret_cast<uint4*>(base + atom * (BK * 128) + row * 128 + ch * 16) = z;
            }
            fence_proxy_async_smem();
          }
          __syncwarp();
        }
        if (lane == 0) {
          const uint32_t a_base = smem_u32(sA);
          const uint32_t b_base = smem_u32(sB);
          // operands read transposed for this k-block (symmetric upper-stored operands)
          const bool kt_left = PAIR && !A_MN && args.sym_ops != 0 && (kb * BK) / TM < ti.mt;
          const bool a_mn = A_MN || (kt_left && (args.sym_ops & 1));
          const bool b_mn = B_MN || (PAIR && !A_MN && (args.sym_ops & 2) && (kb * BK) / TM < ti.nt);
          const uint32_t kid = idesc_f16(TM, BN, DT == ZS_BF16 ? 1u : 0u, a_mn ? 1u : 0u, b_mn ? 1u : 0u);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t adesc = a_mn ? smem_desc(a_base + kk * 2048, BK * 128, 1024, 2)
                                        : smem_desc(a_base + kk * 32, 16, 1024, 2);
            const uint64_t bdesc = b_mn ? smem_desc(b_base + kk * 2048, BK * 128, 1024, 2)
                                        : smem_desc(b_base + kk * 32, 16, 1024, 2);
            const uint32_t use_id = (A_MN == a_mn && B_MN == b_mn) ? idesc : kid;
            if (PAIR)
              tc_mma_f16_pair(d_tmem, adesc, bdesc, use_id, (kb > 0 || kk > 0) ? 1u : 0u);
            else
              tc_mma_f16(d_tmem, adesc, bdesc, use_id, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          if (PAIR)
            tc_commit_pair(&empty[stage], 0x3);
          else
            tc_commit(&empty[stage]);
          issued_any = true;
        }
        __syncwarp();
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      if (lane == 0) {
        if (PAIR)
          tc_commit_pair(&tfull[buf], 0x3);
        else
          tc_commit(&tfull[buf]);
      }
      __syncwarp();
      ++acc_iter;
    }
    // Make sure every MMA this thread issued has finished before TMEM is freed.
    if (lane == 0 && issued_any) {
      if (PAIR)
        tc_commit_pair(done, 0x1);
      else
        tc_commit(done);
      mbar_wait(done, 0, nullptr, ZS_DEVERR_TIMEOUT_DRAIN);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    // 8 warps: warp w reads TMEM lane quarter (w % 4) (rows 32q..32q+31 of
    // the tile) and one half of the tile's columns, h = (w - 2) / 4.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in_tile = quarter * 32 + lane;
    uint8_t* stg = smem + L::OFF_STG + (warp - 2) * STG_BYTES;
    const bool vec = args.vec_ok;
    uint32_t acc_iter = 0;
    for (int t = t_first; t < total_tiles; t += t_step) {
      const TileInfo ti = decode_tile<BN, TM>(t, args, s_tprefix, s_rstart, s_order);
      if (args.mode == MODE_XTY && ti.nkb == 0) {
        // Expert without rows: its weight gradient is zero.
        const int m = ti.mt * BM + row_in_tile;
        float z[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) z[j] = 0.f;
        for (int c = 0; c < BN / 64; ++c) {
          const int col0 = ti.nt * BN + half * (BN / 2) + c * 32;
          const int ncols = min(32, args.N_out - col0);
          if (ncols <= 0) break;
          const int64_t roff = ti.e * args.out_se + (int64_t)m * args.ldo_m;
          if (EPI == EPI_F32) {
            uint32_t zr[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) zr[j] = 0u;
            if (m < args.M_xty)
              store_f32_chunk(reinterpret_cast<float*>(args.out) + roff + col0, zr, ncols, args.accumulate != 0, vec);
          } else {
            emit_chunk<DT>(args.out, roff, col0, ncols, m < args.M_xty, z, vec, stg);
          }
        }
        continue;
      }
      const uint32_t buf = acc_iter & 1;
      const uint32_t acc_phase = (acc_iter >> 1) & 1;
      // Row bookkeeping and (EPI_DSWIGLU) the saved-activation loads do not
      // depend on the accumulator: issue them before waiting for the MMA.
      const int row = ti.r0 + (int)crank * BM + row_in_tile;
      int64_t out_row = row;
      bool valid = args.mode == MODE_ROWS && row < ti.r1;
      if (valid && args.row_map != nullptr) {
        out_row = __ldg(args.row_map + row);
        if (out_row < 0 || out_row >= args.out_rows) {
          record_error(ZS_DEVERR_INDEX);
          valid = false;
        }
      }
      uint4 hcur[4], gcur[4];
      if (EPI == EPI_DSWIGLU) prefetch_chunk(args, out_row, ti.nt * BN + half * (BN / 2), valid && vec, hcur, gcur);
      if (!warp_wait(&tfull[buf], acc_phase, s_abort, ZS_DEVERR_TIMEOUT_EPILOGUE)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + buf * BN;
      // this warp's 32 output rows go out by TMA stores when all of them belong to the tile
      const int crow0 = ti.r0 + (int)crank * BM + quarter * 32;
      const bool tchunk = (EPI == EPI_STORE || EPI == EPI_AXPBY) && args.mode == MODE_ROWS && args.tma_store &&
                          vec && crow0 + 32 <= ti.r1;

      if (args.mode == MODE_ROWS) {
        if (EPI == EPI_SWIGLU) {
          // D columns [0, BN/2) hold the "up" half, [BN/2, BN) the "gate"
          // half; this warp produces activation columns [h*BN/4, (h+1)*BN/4).
#pragma unroll 1
          for (int c = 0; c < BN / 128; ++c) {
            const int lc = half * (BN / 4) + c * 32;
            uint32_t ru[32], rg[32];
            tmem_ld_32x32b_x32(t_row + lc, ru);
            tmem_ld_32x32b_x32(t_row + BN / 2 + lc, rg);
            tc_wait_ld();
            const int col0 = ti.nt * (BN / 2) + lc;
            const int ncols = min(32, args.N_out - col0);
            if (ncols <= 0) continue;
            // u, g as stored (rounded), act = round(round(silu(g)) * u)
            uint32_t pu[16], pg[16], pa[16];
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
              pu[jj] = pk<DT>(__uint_as_float(ru[2 * jj]), __uint_as_float(ru[2 * jj + 1]));
              pg[jj] = pk<DT>(__uint_as_float(rg[2 * jj]), __uint_as_float(rg[2 * jj + 1]));
              const float2 g2 = unpk<DT>(pg[jj]);
              pa[jj] = mul_rn<DT>(pk<DT>(silu_fast(g2.x), silu_fast(g2.y)), pu[jj]);
            }
            emit_packed<DT>(args.out, out_row * args.ldo_m, col0, ncols, valid, pa, vec, stg);
            if (args.out2 != nullptr) {
              emit_packed<DT>(args.out2, out_row * args.ldo2, col0, ncols, valid, pu, vec, stg);
              emit_packed<DT>(args.out2, out_row * args.ldo2, args.swiglu_half + col0, ncols, valid, pg, vec, stg);
            }
          }
        } else if (EPI == EPI_DSWIGLU) {
          // The accumulator is d(act) for activation columns; combine it with
          // the saved pre-activation [h | g] into d[h | g] in one pass, with
          // the reference's rounding points:
          //   dh = round(da * round(silu(g))),  dg = round(round(da * h) * silu'(g))
          // Both halves of the next chunk are fetched during this one (the first
          // chunk's before the accumulator wait).
#pragma unroll 1
          for (int c = 0; c < BN / 64; ++c) {
            const int lc = half * (BN / 2) + c * 32;
            uint4 hnext[4], gnext[4];
            prefetch_chunk(args, out_row, ti.nt * BN + lc + 32, valid && vec && c + 1 < BN / 64, hnext, gnext);
            const int col0 = ti.nt * BN + lc;
            const int ncols = min(32, args.N_out - col0);
            uint4 hraw[4];
            const bool fast = vec && ncols == 32;
#pragma unroll
            for (int q = 0; q < 4; ++q) hraw[q] = hcur[q];
            uint32_t r[32];
            tmem_ld_32x32b_x32(t_row + lc, r);
            tc_wait_ld();
            if (ncols <= 0) continue;
            if (!fast) {
              // ragged edge: plain loads
              float hv[32], gv[32];
              load_chunk(args.aux, out_row * args.ld_aux, col0, ncols, valid, hv, DT, vec);
              load_chunk(args.aux, out_row * args.ld_aux, args.swiglu_half + col0, ncols, valid, gv, DT, vec);
              uint32_t ph[16], pgv[16];
#pragma unroll
              for (int jj = 0; jj < 16; ++jj) {
                ph[jj] = pk<DT>(hv[2 * jj], hv[2 * jj + 1]);
                pgv[jj] = pk<DT>(gv[2 * jj], gv[2 * jj + 1]);
              }
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                hraw[q] = make_uint4(ph[4 * q], ph[4 * q + 1], ph[4 * q + 2], ph[4 * q + 3]);
                gcur[q] = make_uint4(pgv[4 * q], pgv[4 * q + 1], pgv[4 * q + 2], pgv[4 * q + 3]);
              }
            }
            uint32_t odh[16], odg[16];
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
              const uint32_t da = pk<DT>(__uint_as_float(r[2 * jj]), __uint_as_float(r[2 * jj + 1]));
              const uint32_t gw = word_of(gcur, jj);
              const float2 g2 = unpk<DT>(gw);
              const float s0 = sigmoid_fast(g2.x), s1 = sigmoid_fast(g2.y);
              odh[jj] = mul_rn<DT>(da, pk<DT>(g2.x * s0, g2.y * s1));
              const float2 t2 = unpk<DT>(mul_rn<DT>(da, word_of(hraw, jj)));
              odg[jj] = pk<DT>(t2.x * (s0 * (1.0f + g2.x * (1.0f - s0))), t2.y * (s1 * (1.0f + g2.y * (1.0f - s1))));
            }
            emit_packed<DT>(args.out, out_row * args.ldo_m, col0, ncols, valid, odh, vec, stg);
            emit_packed<DT>(args.out, out_row * args.ldo_m, args.swiglu_half + col0, ncols, valid, odg, vec, stg);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              hcur[q] = hnext[q];
              gcur[q] = gnext[q];
            }
          }
        } else if (EPI == EPI_LSE || EPI == EPI_XENT_GRAD) {
          // Columns are vocabulary entries col_offset + col.  Labels of this
          // row, relative to this warp's first column, found by range test.
          int si = 0;
          int64_t lab[8];
          const int64_t wcol = args.col_offset + ti.nt * BN + half * (BN / 2);
          if (valid) {
            si = min(__ldg(args.s_count + row), args.s_max);
#pragma unroll
            for (int j = 0; j < 8; ++j) lab[j] = (j < si) ? __ldg(args.labels + (int64_t)row * args.s_max + j) - wcol : -1;
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) lab[j] = -1;
          }
          float run_m = -INFINITY, run_s = 0.f, tgt = 0.f;
          float alpha = 0.f, scale = 0.f, lrow = 0.f;
          if (EPI == EPI_XENT_GRAD) {
            // G = s * softmax - counts, unscaled: grad_loss / N is applied in f32 by the dH and
            // dW products (a bf16 G of (softmax - 1) / N would round every row's target entry
            // the same way and scale the whole gradient by up to 2^-8)
            scale = 1.0f;
            alpha = (float)si;
            lrow = valid ? __ldg(args.lse + row) : 0.f;
          }
#pragma unroll 1
          for (int c = 0; c < BN / 64; ++c) {
            const int lc = half * (BN / 2) + c * 32;
            uint32_t r[32];
            tmem_ld_32x32b_x32(t_row + lc, r);
            tc_wait_ld();
            const int col0 = ti.nt * BN + lc;
            const int ncols = min(32, args.N_out - col0);
            if (ncols <= 0) continue;
            if (EPI == EPI_LSE) {
              float cm = -INFINITY;
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (j < ncols) cm = fmaxf(cm, __uint_as_float(r[j]));
              const float nm = fmaxf(run_m, cm);
              float acc = run_s * __expf(run_m - nm);
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (j < ncols) acc += __expf(__uint_as_float(r[j]) - nm);
              run_m = nm;
              run_s = acc;
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const int64_t off = lab[j] - c * 32;
                if (off >= 0 && off < ncols) {
                  float z = 0.f;
#pragma unroll
                  for (int q = 0; q < 32; ++q) z = (q == (int)off) ? __uint_as_float(r[q]) : z;
                  tgt += z;
                }
              }
            } else {
              float g[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) g[j] = alpha * __expf(__uint_as_float(r[j]) - lrow);
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const int64_t off = lab[j] - c * 32;
                if (off >= 0 && off < ncols) {
#pragma unroll
                  for (int q = 0; q < 32; ++q)
                    if (q == (int)off) g[q] -= scale;
                }
              }
              emit_chunk<DT>(args.out, (int64_t)row * args.ldo_m, col0, ncols, valid, g, vec, stg);
            }
          }
          if (EPI == EPI_LSE && valid) {
            const int64_t slot = (int64_t)row * args.part_ld + (int64_t)ti.nt * 2 + half;
            args.part_max[slot] = run_m;
            args.part_sum[slot] = run_s;
            if (tgt != 0.f) atomicAdd(args.target_sum + row, tgt);
          }
        } else if (EPI == EPI_AXPBY) {
          // the aux row's next 32 columns are fetched (raw) while this chunk is combined
          auto fetch_aux = [&](int cc, uint4 (&w)[4]) {
            const int c0 = ti.nt * BN + half * (BN / 2) + cc * 32;
            const bool ok = valid && vec && cc < BN / 64 && c0 + 32 <= args.N_out;
            const uint4* p = reinterpret_cast<const uint4*>(args.aux + (out_row * args.ld_aux + c0) * 2);
#pragma unroll
            for (int q = 0; q < 4; ++q) w[q] = ok ? __ldg(p + q) : make_uint4(0, 0, 0, 0);
          };
          uint4 acur[4];
          fetch_aux(0, acur);
#pragma unroll 1
          for (int c = 0; c < BN / 64; ++c) {
            const int lc = half * (BN / 2) + c * 32;
            const int col0 = ti.nt * BN + lc;
            const int ncols = min(32, args.N_out - col0);
            uint4 anext[4];
            fetch_aux(c + 1, anext);
            float av[32];
            if (vec && ncols == 32) {
#pragma unroll
              for (int jj = 0; jj < 16; ++jj) {
                const float2 f = unpk<DT>(word_of(acur, jj));
                av[2 * jj] = valid ? f.x : 0.f;
                av[2 * jj + 1] = valid ? f.y : 0.f;
              }
            } else if (ncols > 0) {
              load_chunk(args.aux, out_row * args.ld_aux, col0, ncols, valid, av, DT, vec);
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) acur[q] = anext[q];
            uint32_t r[32];
            tmem_ld_32x32b_x32(t_row + lc, r);
            tc_wait_ld();
            if (ncols <= 0) continue;
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = fmaf(args.alpha, __uint_as_float(r[j]), args.beta * av[j]);
            uint32_t pv[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) pv[j] = pack2(v[2 * j], v[2 * j + 1], DT);
            if (tchunk && ncols == 32) {
              tma_emit_chunk(&tmO, stg, pv, col0, crow0, false);
            } else {
              if (args.tma_store && lane == 0) bulk_wait_read_all();   // staging buffer free
              __syncwarp();
              emit_packed<DT>(args.out, out_row * args.ldo_m, col0, ncols, valid, pv, vec, stg);
            }
            if (args.sym_upper && !args.sym_ops && ti.mt < ti.nt) {
              const int64_t gbase = ti.r0 - (int64_t)ti.mt * TM;   // first row of this square group
              if (tchunk && ncols == 32)
                tma_emit_chunk(&tmO, stg, pv, (int)(ti.r0 - gbase) + (int)crank * BM + quarter * 32,
                               (int)(gbase + col0), true);
              else
                emit_packed_mirror(args.out, args.ldo_m, gbase + col0,
                                   ti.r0 - gbase + (int)crank * BM + quarter * 32, pv, stg);
            }
          }
        } else if (EPI == EPI_F32) {
#pragma unroll 1
          for (int c = 0; c < BN / 64; ++c) {
            const int lc = half * (BN / 2) + c * 32;
            uint32_t r[32];
            tmem_ld_32x32b_x32(t_row + lc, r);
            tc_wait_ld();
            const int col0 = ti.nt * BN + lc;
            const int ncols = min(32, args.N_out - col0);
            if (ncols <= 0 || !valid) continue;
            if (args.f32_scale != nullptr) {
              const float sc = __ldg(args.f32_scale);
#pragma unroll
              for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * sc);
            }
            float* o = reinterpret_cast<float*>(args.out) + out_row * args.ldo_m + col0;
            store_f32_chunk(o, r, ncols, args.accumulate != 0, vec);
          }
        } else {
#pragma unroll 1
          for (int c = 0; c < BN / 64; ++c) {
            const int lc = half * (BN / 2) + c * 32;
            uint32_t r[32];
            tmem_ld_32x32b_x32(t_row + lc, r);
            tc_wait_ld();
            const int col0 = ti.nt * BN + lc;
            const int ncols = min(32, args.N_out - col0);
            if (ncols <= 0) continue;
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
            if (args.bias != nullptr && valid) {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                if (j < ncols) {
                  const int64_t bi = ti.e * args.bias_se + (int64_t)(col0 + j) * args.bias_sn;
                  v[j] += DT == ZS_BF16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(args.bias)[bi])
                                        : __half2float(reinterpret_cast<const __half*>(args.bias)[bi]);
                }
              }
            }
            uint32_t pv[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) pv[j] = pack2(v[2 * j], v[2 * j + 1], DT);
            if (tchunk && ncols == 32) {
              tma_emit_chunk(&tmO, stg, pv, col0, crow0, false);
            } else {
              if (args.tma_store && lane == 0) bulk_wait_read_all();
              __syncwarp();
              emit_packed<DT>(args.out, out_row * args.ldo_m, col0, ncols, valid, pv, vec, stg);
            }
            if (args.sym_upper && !args.sym_ops && ti.mt < ti.nt) {
              const int64_t gbase = ti.r0 - (int64_t)ti.mt * TM;
              if (tchunk && ncols == 32)
                tma_emit_chunk(&tmO, stg, pv, (int)(ti.r0 - gbase) + (int)crank * BM + quarter * 32,
                               (int)(gbase + col0), true);
              else
                emit_packed_mirror(args.out, args.ldo_m, gbase + col0,
                                   ti.r0 - gbase + (int)crank * BM + quarter * 32, pv, stg);
            }
          }
        }
      } else {
        const int m = ti.mt * BM + row_in_tile;
        const bool mvalid = m < args.M_xty;
#pragma unroll 1
        for (int c = 0; c < BN / 64; ++c) {
          const int lc = half * (BN / 2) + c * 32;
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + lc, r);
          tc_wait_ld();
          const int col0 = ti.nt * BN + lc;
          const int ncols = min(32, args.N_out - col0);
          if (ncols <= 0) continue;
          if (EPI == EPI_F32) {
            if (mvalid) {
              if (args.f32_scale != nullptr) {
                const float sc = __ldg(args.f32_scale);
#pragma unroll
                for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * sc);
              }
              float* o = reinterpret_cast<float*>(args.out) + ti.e * args.out_se + (int64_t)m * args.ldo_m + col0;
              store_f32_chunk(o, r, ncols, args.accumulate != 0, vec);
            }
            continue;
          }
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
          emit_chunk<DT>(args.out, ti.e * args.out_se + (int64_t)m * args.ldo_m, col0, ncols, mvalid, v, vec, stg);
        }
      }
      // every lane's TMEM reads of this buffer are complete (tcgen05.wait::ld
      // after each load); one arrival per warp releases it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR)
          mbar_arrive_cluster(&tempty[buf], 0);
        else
          mbar_arrive(&tempty[buf]);
      }
      ++acc_iter;
    }
    // the TMA stores issued from this warp's staging buffer have completed
    if (args.tma_store && lane == 0) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  // a pair stays resident until neither CTA touches the other's shared memory
  // (rank 0's MMAs read rank 1's operands; rank 1 arrives on rank 0's barriers)
  if (PAIR) cluster_sync_all();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    if (PAIR)
      tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else
      tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host side

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D bf16/f16 tensor map with 128-byte swizzle.  inner/outer are the extents
// in elements/rows, row_bytes the row pitch.
static int make_tmap(CUtensorMap* m, const void* base, int dtype, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                     uint32_t box_inner, uint32_t box_outer,
                     CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto fn = encode_fn();
  if (fn == nullptr) return ZS_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return ZS_ERR_ALIGN;
  if ((row_bytes & 15) != 0) return ZS_ERR_ALIGN;
  if (inner == 0 || outer == 0) return ZS_ERR_SHAPE;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, dtype == ZS_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                  const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    zs_last_cuda_error_ref() = 100000 + (int)r;  // driver result codes, offset
    return ZS_ERR_CUDA;
  }
  return ZS_OK;
}

// Tensor map of a 16-bit output [rows, cols] (row pitch row_bytes) for the
// TMA-store epilogue: 32 x 32 boxes, 64-byte swizzle.
static int make_out_tmap(CUtensorMap* m, const void* base, int dtype, uint64_t cols, uint64_t rows,
                         uint64_t row_bytes) {
  return make_tmap(m, base, dtype, cols, rows, row_bytes, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
}

static int& gemm_cta_limit_ref() {
  static int lim = 0;
  return lim;
}
int zs_gemm_cta_limit() { return gemm_cta_limit_ref(); }

int num_sms() {
  static int n = 0;
  static int dev_cached = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != dev_cached) {
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    dev_cached = dev;
  }
  return n > 0 ? n : 148;
}

// Newton-Schulz keeps only the upper tiles of its symmetric products unless
// ZS_NS_MIRROR=1 in the environment asks for whole matrices (mirrored tiles).
static bool sym_operands_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* e = getenv("ZS_NS_MIRROR");
    on = (e != nullptr && e[0] == '1') ? 0 : 1;
  }
  return on == 1;
}

// Pair (2-SM) tiles are used for MODE_ROWS unless disabled with
// ZS_GEMM_PAIR=0 in the environment, or the groups are uniform and shorter
// than a pair tile (small batched matrices waste less with 128-row tiles).
static bool pair_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* e = getenv("ZS_GEMM_PAIR");
    on = (e != nullptr && e[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

template <int BN, bool A_MN, bool B_MN, int EPI, int DT>
static int launch_pair(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmO,
                       const CUtensorMap& tmAT, const CUtensorMap& tmBT, const GemmArgs& args, int64_t max_tiles,
                       cudaStream_t stream) {
  constexpr int STAGES = 6;
  using L = Smem<BN, STAGES, true>;
  auto kern = grouped_gemm_kernel<BN, STAGES, A_MN, B_MN, EPI, DT, true>;
  static int max_clusters = -1;   // per instantiation
  if (max_clusters < 0) {
    ZS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC));
    cudaLaunchConfig_t q = {};
    cudaLaunchAttribute qa[1];
    qa[0].id = cudaLaunchAttributeClusterDimension;
    qa[0].val.clusterDim.x = 2;
    qa[0].val.clusterDim.y = 1;
    qa[0].val.clusterDim.z = 1;
    q.gridDim = dim3(2 * (unsigned)(num_sms() / 2));
    q.blockDim = dim3(64 + 32 * NUM_EPI_WARPS);
    q.dynamicSmemBytes = L::ALLOC;
    q.attrs = qa;
    q.numAttrs = 1;
    int n = 0;
    ZS_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, kern, &q));
    max_clusters = n;
  } else {
    ZS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC));
  }
  // persistent: no more clusters than can be resident at once
  int64_t clusters = max_clusters;
  const int lim = zs_gemm_cta_limit();
  if (lim > 0 && clusters > lim / 2) clusters = lim / 2;
  if (max_tiles < clusters) clusters = max_tiles;
  if (clusters < 1) clusters = 1;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3((unsigned)(2 * clusters));
  cfg.blockDim = dim3(64 + 32 * NUM_EPI_WARPS);
  cfg.dynamicSmemBytes = L::ALLOC;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  ZS_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, tmA, tmB, tmO, tmAT, tmBT, args));
  return ZS_OK;
}

// tmO: the output's tensor map for the TMA-store epilogue (args.tma_store), else unused.
template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI>
// tmAT / tmBT: MN-major maps of symmetric operands stored as upper tiles (args.sym_ops).
static int launch_gemm(const CUtensorMap& tmA, const CUtensorMap& tmB, const GemmArgs& args, int64_t max_tiles,
                       cudaStream_t stream, const CUtensorMap* tmO = nullptr, const CUtensorMap* tmAT = nullptr,
                       const CUtensorMap* tmBT = nullptr) {
  const CUtensorMap& tO = tmO != nullptr ? *tmO : tmA;
  const CUtensorMap& tAT = tmAT != nullptr ? *tmAT : tmA;
  const CUtensorMap& tBT = tmBT != nullptr ? *tmBT : tmB;
  if (args.tma_store && tmO == nullptr) return ZS_ERR_ARG;
  if (((args.sym_ops & 1) && tmAT == nullptr) || ((args.sym_ops & 2) && tmBT == nullptr)) return ZS_ERR_ARG;
  if constexpr (!A_MN) {
    if (args.mode == MODE_ROWS && pair_enabled() && !(args.group_rows > 0 && args.group_rows < 2 * BM)) {
      return args.out_dtype == ZS_F16
                 ? launch_pair<BN, A_MN, B_MN, EPI, ZS_F16>(tmA, tmB, tO, tAT, tBT, args, max_tiles, stream)
                 : launch_pair<BN, A_MN, B_MN, EPI, ZS_BF16>(tmA, tmB, tO, tAT, tBT, args, max_tiles, stream);
    }
  }
  using L = Smem<BN, STAGES>;
  auto kern = args.out_dtype == ZS_F16 ? grouped_gemm_kernel<BN, STAGES, A_MN, B_MN, EPI, ZS_F16, false>
                                       : grouped_gemm_kernel<BN, STAGES, A_MN, B_MN, EPI, ZS_BF16, false>;
  ZS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC));
  int64_t grid = num_sms();
  // leave SMs free for kernels that must run alongside (a collective on another stream)
  const int lim = zs_gemm_cta_limit();
  if (lim > 0 && grid > lim) grid = lim;
  if (max_tiles < grid) grid = max_tiles;
  if (grid < 1) grid = 1;
  if (args.sym_ops) return ZS_ERR_ARG;   // symmetric operands need pair tiles
  kern<<<(unsigned)grid, 64 + 32 * NUM_EPI_WARPS, L::ALLOC, stream>>>(tmA, tmB, tO, tAT, tBT, args);
  ZS_CUDA_TRY(cudaGetLastError());
  return ZS_OK;
}

}  // namespace zs

// Declared in zs_moe.cu.
namespace zs {
int launch_group(const void* A, int64_t a_sm, int64_t K, void* Y, int64_t y_sm, int64_t n, const void* coeff,
                 int coeff_dtype, int fan_out, const int64_t* ssi, int dtype, cudaStream_t stream);
}

using namespace zs;

static inline int elem_size(int dtype) { return dtype == ZS_F32 ? 4 : 2; }

extern "C" size_t zs_scatter2scatter_workspace(int64_t n, int64_t K, int dtype, int x_grouped) {
  if (x_grouped) return 0;
  // gathered rows, padded so the row pitch is a multiple of 16 bytes
  const int64_t pitch = ((K * elem_size(dtype) + 15) / 16) * 16;
  return (size_t)(n * pitch + 256);
}

extern "C" int zs_scatter2scatter(void* out, int64_t out_sm, const void* W, int64_t num_experts, int64_t K,
                                  int64_t N, int64_t w_se, int64_t w_sk, int64_t w_sn, const void* X, int64_t x_rows,
                                  int64_t x_sm, const void* bias, int64_t b_se, int64_t b_sn, int fan_out,
                                  const int64_t* sorted_expert_idxs, const int64_t* sorted_scattered_idxs,
                                  const int64_t* expert_offsets, int64_t n, int x_grouped, int y_grouped, int dtype,
                                  void* workspace, size_t workspace_bytes, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ZS_REQUIRE(out && W && X && sorted_expert_idxs && sorted_scattered_idxs, ZS_ERR_ARG);
  ZS_REQUIRE(dtype == ZS_BF16 || dtype == ZS_F16, ZS_ERR_DTYPE);
  ZS_REQUIRE(num_experts >= 1 && num_experts <= MAX_EXPERTS_GEMM, ZS_ERR_SHAPE);
  ZS_REQUIRE(K >= 1 && N >= 1 && n >= 0 && fan_out >= 1, ZS_ERR_SHAPE);
  ZS_REQUIRE(n < (int64_t)1 << 30 && K < (int64_t)1 << 24 && N < (int64_t)1 << 24, ZS_ERR_SHAPE);
  ZS_REQUIRE(x_grouped ? (x_rows == n) : (x_rows * fan_out == n), ZS_ERR_SHAPE);
  ZS_BIND(X);
  if (n == 0) return ZS_OK;
  const int es = elem_size(dtype);

  // B operand layout
  bool b_mn;
  if (w_sk == 1 && w_se == N * w_sn && w_sn >= K)
    b_mn = false;
  else if (w_sn == 1 && w_se == K * w_sk && w_sk >= N)
    b_mn = true;
  else
    return ZS_ERR_LAYOUT;

  // A operand: grouped rows, gathered into the workspace when needed
  const void* A = X;
  int64_t a_sm = x_sm;
  if (!x_grouped) {
    const size_t need = zs_scatter2scatter_workspace(n, K, dtype, 0);
    ZS_REQUIRE(workspace != nullptr && workspace_bytes >= need, ZS_ERR_WORKSPACE);
    char* ws = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
    const int64_t pitch = ((K * es + 15) / 16) * 16 / es;
    int rc = launch_group(X, x_sm, K, ws, pitch, n, nullptr, dtype, fan_out, sorted_scattered_idxs, dtype, stream);
    if (rc != ZS_OK) return rc;
    A = ws;
    a_sm = pitch;
  }

  CUtensorMap tmA, tmB;
  int rc = make_tmap(&tmA, A, dtype, (uint64_t)K, (uint64_t)n, (uint64_t)a_sm * es, 64, 128);
  if (rc != ZS_OK) return rc;
  constexpr int BN = 256;
  if (!b_mn)
    rc = make_tmap(&tmB, W, dtype, (uint64_t)K, (uint64_t)(num_experts * N), (uint64_t)w_sn * es, 64, BN / 2);
  else
    rc = make_tmap(&tmB, W, dtype, (uint64_t)N, (uint64_t)(num_experts * K), (uint64_t)w_sk * es, 64, 64);
  if (rc != ZS_OK) return rc;

  GemmArgs a{};
  a.mode = MODE_ROWS;
  a.num_experts = (int)num_experts;
  a.n_tiles = (int)((N + BN - 1) / BN);
  a.kb_rows = (int)((K + BK - 1) / BK);
  a.N_out = (int)N;
  a.ab_fmt = dtype == ZS_BF16 ? 1 : 0;
  a.n_rows = n;
  a.expert_offsets = expert_offsets;
  a.sorted_expert_idxs = sorted_expert_idxs;
  a.row_map = y_grouped ? nullptr : sorted_scattered_idxs;
  a.out_rows = n;
  a.out = reinterpret_cast<char*>(out);
  a.ldo_m = out_sm;
  a.ldo_n = 1;
  a.bias = reinterpret_cast<const char*>(bias);
  a.bias_se = b_se;
  a.bias_sn = b_sn;
  a.out_dtype = dtype;
  a.b_rows_per_expert = (int)(b_mn ? K : N);
  a.vec_ok = ((reinterpret_cast<uintptr_t>(out) & 15) == 0) && ((out_sm * es) % 16 == 0);
  const int64_t max_tiles = (n / BM + num_experts) * a.n_tiles;
  // grouped output rows without a bias: full chunks go out by TMA stores
  CUtensorMap tmO;
  if (y_grouped && bias == nullptr && a.vec_ok &&
      make_out_tmap(&tmO, out, dtype, (uint64_t)N, (uint64_t)n, (uint64_t)out_sm * es) == ZS_OK)
    a.tma_store = 1;
  const CUtensorMap* pO = a.tma_store ? &tmO : nullptr;
  if (!b_mn) return launch_gemm<BN, 4, false, false, EPI_STORE>(tmA, tmB, a, max_tiles, stream, pO);
  return launch_gemm<BN, 4, false, true, EPI_STORE>(tmA, tmB, a, max_tiles, stream, pO);
}

extern "C" int zs_group_xty(int num_experts, void* DW, int64_t dw_se, int64_t dw_sk, int64_t dw_sn, void* Db,
                            int64_t db_se, int64_t db_sn, const void* DY, int64_t dy_sm, const void* X, int64_t x_sm,
                            int64_t n, int64_t K, int64_t N, const int64_t* expert_offsets, int dtype,
                            void* stream_);

namespace zs {
int launch_colsum_per_expert(void* Db, int64_t db_se, int64_t db_sn, const void* DY, int64_t dy_sm, int64_t N,
                             int num_experts, const int64_t* expert_offsets, int dtype, cudaStream_t stream);
}

namespace zs {
// DW[e] = X_e^T DY_e for every expert; EPI_STORE writes the input dtype,
// EPI_F32 writes (or with accumulate adds into) f32.
template <int EPI>
static int group_xty_impl(int num_experts, void* DW, int64_t dw_se, int64_t dw_sk, int64_t dw_sn, const void* DY,
                          int64_t dy_sm, const void* X, int64_t x_sm, int64_t n, int64_t K, int64_t N,
                          const int64_t* expert_offsets, int dtype, int accumulate, cudaStream_t stream) {
  const int es = elem_size(dtype);
  const int oes = EPI == EPI_F32 ? 4 : es;
  constexpr int BN = 256;

  // Orientation: GEMM rows m run along the stride-1 side when possible so the
  // epilogue writes 16-byte row segments.
  //   dw_sn == 1: m = k (A = X^T), n = n (B = DY^T), element at m*dw_sk + n
  //   dw_sk == 1: m = n (A = DY^T), n = k (B = X^T), element at m*dw_sn + k
  bool swap;
  if (dw_sn == 1)
    swap = false;
  else if (dw_sk == 1)
    swap = true;
  else
    return ZS_ERR_LAYOUT;
  const void* Aop = swap ? DY : X;
  const int64_t a_sm = swap ? dy_sm : x_sm;
  const int64_t Mext = swap ? N : K;
  const void* Bop = swap ? X : DY;
  const int64_t b_sm = swap ? x_sm : dy_sm;
  const int64_t Next = swap ? K : N;

  GemmArgs a{};
  a.mode = MODE_XTY;
  a.num_experts = num_experts;
  a.n_tiles = (int)((Next + BN - 1) / BN);
  a.m_tiles_xty = (int)((Mext + BM - 1) / BM);
  a.M_xty = (int)Mext;
  a.N_out = (int)Next;
  a.ab_fmt = dtype == ZS_BF16 ? 1 : 0;
  a.n_rows = n;
  a.expert_offsets = expert_offsets;
  a.out = reinterpret_cast<char*>(DW);
  a.ldo_m = swap ? dw_sn : dw_sk;
  a.ldo_n = 1;
  a.out_se = dw_se;
  a.out_dtype = dtype;
  a.accumulate = accumulate;
  a.vec_ok = ((reinterpret_cast<uintptr_t>(DW) & 15) == 0) && ((a.ldo_m * oes) % 16 == 0) &&
             ((dw_se * oes) % 16 == 0);

  const int64_t max_tiles = (int64_t)num_experts * a.m_tiles_xty * a.n_tiles;
  if (n == 0) {
    // every expert is empty: the kernel only writes zeros; TMA maps need a
    // nonzero extent, so point them at a 1-row view of the (unused) inputs.
    n = 1;
  }
  CUtensorMap tmA, tmB;
  int rc = make_tmap(&tmA, Aop, dtype, (uint64_t)Mext, (uint64_t)n, (uint64_t)a_sm * es, 64, 64);
  if (rc != ZS_OK) return rc;
  rc = make_tmap(&tmB, Bop, dtype, (uint64_t)Next, (uint64_t)n, (uint64_t)b_sm * es, 64, 64);
  if (rc != ZS_OK) return rc;
  return launch_gemm<BN, 4, true, true, EPI>(tmA, tmB, a, max_tiles, stream);
}
}  // namespace zs

extern "C" int zs_group_xty(int num_experts, void* DW, int64_t dw_se, int64_t dw_sk, int64_t dw_sn, void* Db,
                            int64_t db_se, int64_t db_sn, const void* DY, int64_t dy_sm, const void* X, int64_t x_sm,
                            int64_t n, int64_t K, int64_t N, const int64_t* expert_offsets, int dtype,
                            void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ZS_REQUIRE(DW && DY && X && expert_offsets, ZS_ERR_ARG);
  ZS_REQUIRE(dtype == ZS_BF16 || dtype == ZS_F16, ZS_ERR_DTYPE);
  ZS_REQUIRE(num_experts >= 1 && num_experts <= MAX_EXPERTS_GEMM, ZS_ERR_SHAPE);
  ZS_REQUIRE(K >= 1 && N >= 1 && n >= 0, ZS_ERR_SHAPE);
  ZS_REQUIRE(n < (int64_t)1 << 30 && K < (int64_t)1 << 24 && N < (int64_t)1 << 24, ZS_ERR_SHAPE);
  ZS_BIND(DY);
  int rc = group_xty_impl<EPI_STORE>(num_experts, DW, dw_se, dw_sk, dw_sn, DY, dy_sm, X, x_sm, n, K, N,
                                     expert_offsets, dtype, 0, stream);
  if (rc != ZS_OK) return rc;
  if (Db != nullptr)
    rc = launch_colsum_per_expert(Db, db_se, db_sn, DY, dy_sm, N, num_experts, expert_offsets, dtype, stream);
  return rc;
}

extern "C" int zs_set_gemm_cta_limit(int max_ctas) {
  ZS_REQUIRE(max_ctas >= 0, ZS_ERR_ARG);
  gemm_cta_limit_ref() = max_ctas;
  return ZS_OK;
}

extern "C" int zs_group_xty_f32(int num_experts, float* DW, int64_t dw_se, int64_t dw_sk, int64_t dw_sn,
                                const void* DY, int64_t dy_sm, const void* X, int64_t x_sm, int64_t n, int64_t K,
                                int64_t N, const int64_t* expert_offsets, int dtype, int accumulate, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ZS_REQUIRE(DW && DY && X && expert_offsets, ZS_ERR_ARG);
  ZS_REQUIRE(dtype == ZS_BF16 || dtype == ZS_F16, ZS_ERR_DTYPE);
  ZS_REQUIRE(num_experts >= 1 && num_experts <= MAX_EXPERTS_GEMM, ZS_ERR_SHAPE);
  ZS_REQUIRE(K >= 1 && N >= 1 && n >= 0, ZS_ERR_SHAPE);
  ZS_REQUIRE(n < (int64_t)1 << 30 && K < (int64_t)1 << 24 && N < (int64_t)1 << 24, ZS_ERR_SHAPE);
  ZS_BIND(DY);
  return group_xty_impl<EPI_F32>(num_experts, DW, dw_se, dw_sk, dw_sn, DY, dy_sm, X, x_sm, n, K, N, expert_offsets,
                                 dtype, accumulate != 0, stream);
}

extern "C" int zs_expert_up_swiglu(void* act, void* hfull, const void* W1, int64_t num_experts, int64_t K, int64_t F,
                                   const void* Xg, int64_t xg_sm, const int64_t* sorted_expert_idxs,
                                   const int64_t* expert_offsets, int64_t n, int dtype, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ZS_REQUIRE(act && W1 && Xg && (sorted_expert_idxs || expert_offsets), ZS_ERR_ARG);
  ZS_REQUIRE(dtype == ZS_BF16 || dtype == ZS_F16, ZS_ERR_DTYPE);
  ZS_REQUIRE(num_experts >= 1 && num_experts <= MAX_EXPERTS_GEMM, ZS_ERR_SHAPE);
  ZS_REQUIRE(K >= 1 && F >= 1 && n >= 0, ZS_ERR_SHAPE);
  ZS_REQUIRE(n < (int64_t)1 << 30 && K < (int64_t)1 << 24 && F < (int64_t)1 << 23, ZS_ERR_SHAPE);
  ZS_REQUIRE(num_experts * 2 * F < ((int64_t)1 << 31), ZS_ERR_SHAPE);
  ZS_BIND(Xg);
  if (n == 0) return ZS_OK;
  const int es = elem_size(dtype);
  constexpr int BN = 256;
  CUtensorMap tmA, tmB;
  int rc = make_tmap(&tmA, Xg, dtype, (uint64_t)K, (uint64_t)n, (uint64_t)xg_sm * es, 64, 128);
  if (rc != ZS_OK) return rc;
  rc = make_tmap(&tmB, W1, dtype, (uint64_t)K, (uint64_t)(num_experts * 2 * F), (uint64_t)K * es, 64, BN / 2);
  if (rc != ZS_OK) return rc;
  GemmArgs a{};
  a.mode = MODE_ROWS;
  a.num_experts = (int)num_experts;
  a.n_tiles = (int)((F + BN / 2 - 1) / (BN / 2));
  a.kb_rows = (int)((K + BK - 1) / BK);
  a.N_out = (int)F;
  a.ab_fmt = dtype == ZS_BF16 ? 1 : 0;
  a.n_rows = n;
  a.expert_offsets = expert_offsets;
  a.sorted_expert_idxs = sorted_expert_idxs;
  a.row_map = nullptr;
  a.out_rows = n;
  a.out = reinterpret_cast<char*>(act);
  a.ldo_m = F;
  a.ldo_n = 1;
  a.out2 = reinterpret_cast<char*>(hfull);
  a.ldo2 = 2 * F;
  a.out_dtype = dtype;
  a.b_rows_per_expert = (int)(2 * F);
  a.swiglu_half = (int)F;
  a.vec_ok = ((reinterpret_cast<uintptr_t>(act) | reinterpret_cast<uintptr_t>(hfull)) % 16 == 0) &&
             ((F * es) % 16 == 0);
  const int64_t max_tiles = (n / BM + num_experts) * a.n_tiles;
  return launch_gemm<BN, 4, false, false, EPI_SWIGLU>(tmA, tmB, a, max_tiles, stream);
}

extern "C" int zs_expert_down_dswiglu(void* dhfull, const void* hfull, const void* W2, int64_t num_experts, int64_t K,
                                      int64_t F, const void* dyg, int64_t dyg_sm, const int64_t* sorted_expert_idxs,
                                      const int64_t* expert_offsets, int64_t n, int dtype, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ZS_REQUIRE(dhfull && hfull && W2 && dyg && (sorted_expert_idxs || expert_offsets), ZS_ERR_ARG);
  ZS_REQUIRE(dtype == ZS_BF16 || dtype == ZS_F16, ZS_ERR_DTYPE);
  ZS_REQUIRE(num_experts >= 1 && num_experts <= MAX_EXPERTS_GEMM, ZS_ERR_SHAPE);
  ZS_REQUIRE(K >= 1 && F >= 1 && n >= 0, ZS_ERR_SHAPE);
  ZS_REQUIRE(n < (int64_t)1 << 30 && K < (int64_t)1 << 24 && F < (int64_t)1 << 23, ZS_ERR_SHAPE);
  ZS_REQUIRE(num_experts * K < ((int64_t)1 << 31), ZS_ERR_SHAPE);
  ZS_BIND(dyg);
  if (n == 0) return ZS_OK;
  const int es = elem_size(dtype);
  constexpr int BN = 256;
  CUtensorMap tmA, tmB;
  int rc = make_tmap(&tmA, dyg, dtype, (uint64_t)K, (uint64_t)n, (uint64_t)dyg_sm * es, 64, 128);
  if (rc != ZS_OK) return rc;
  // W2 [E, K, F] viewed as [E*K rows, F cols]: MN-major B (F contiguous)
  rc = make_tmap(&tmB, W2, dtype, (uint64_t)F, (uint64_t)(num_experts * K), (uint64_t)F * es, 64, 64);
  if (rc != ZS_OK) return rc;
  GemmArgs a{};
  a.mode = MODE_ROWS;
  a.num_experts = (int)num_experts;
  a.n_tiles = (int)((F + BN - 1) / BN);
  a.kb_rows = (int)((K + BK - 1) / BK);
  a.N_out = (int)F;
  a.ab_fmt = dtype == ZS_BF16 ? 1 : 0;
  a.n_rows = n;
  a.out_rows = n;
  a.expert_offsets = expert_offsets;
  a.sorted_expert_idxs = sorted_expert_idxs;
  a.out = reinterpret_cast<char*>(dhfull);
  a.ldo_m = 2 * F;
  a.ldo_n = 1;
  a.aux = reinterpret_cast<const char*>(hfull);
  a.ld_aux = 2 * F;
  a.swiglu_half = (int)F;
  a.out_dtype = dtype;
  a.b_rows_per_expert = (int)K;
  a.vec_ok = ((reinterpret_cast<uintptr_t>(dhfull) | reinterpret_cast<uintptr_t>(hfull)) % 16 == 0) &&
             ((F * es) % 16 == 0);
  const int64_t max_tiles = (n / BM + num_experts) * a.n_tiles;
  return launch_gemm<BN, 4, false, true, EPI_DSWIGLU>(tmA, tmB, a, max_tiles, stream);
}

// ------------------------------------------------------------ cross entropy

namespace zs {

// lse[t] from the (max, sum) partials; row loss s_t * lse_t - target_t.
__global__ void xent_finalize_kernel(const float* __restrict__ part_max, const float* __restrict__ part_sum,
                                     int64_t part_ld, int nparts, const float* __restrict__ target_sum,
                                     const int* __restrict__ s_count, int s_max, int64_t T, float* __restrict__ lse,
                                     float* __restrict__ row_loss) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T; t += warps) {
    float m = -INFINITY;
    for (int p = lane; p < nparts; p += 32) m = fmaxf(m, part_max[t * part_ld + p]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    float sum = 0.f;
    for (int p = lane; p < nparts; p += 32) {
      const float pm = part_max[t * part_ld + p];
      if (pm != -INFINITY) sum += part_sum[t * part_ld + p] * expf(pm - m);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    if (lane == 0) {
      const float l = m + logf(sum);
      lse[t] = l;
      const int si = min(s_count[t], s_max);
      row_loss[t] = si > 0 ? (float)si * l - target_sum[t] : 0.f;
    }
  }
}

// loss = sum(row_loss) / sum(s); one block, fixed reduction order.
__global__ void xent_reduce_kernel(const float* __restrict__ row_loss, const int* __restrict__ s_count, int s_max,
                                   int64_t T, float* __restrict__ loss, float* __restrict__ denom) {
  __shared__ double sh_l[32];
  __shared__ long long sh_n[32];
  double l = 0.0;
  long long n = 0;
  for (int64_t t = threadIdx.x; t < T; t += blockDim.x) {
    l += (double)row_loss[t];
    n += min(s_count[t], s_max);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    l += __shfl_xor_sync(0xffffffffu, l, off);
    n += __shfl_xor_sync(0xffffffffu, n, off);
  }
  if ((threadIdx.x & 31) == 0) {
    sh_l[threadIdx.x >> 5] = l;
    sh_n[threadIdx.x >> 5] = n;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double L = 0.0;
    long long N = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
      L += sh_l[w];
      N += sh_n[w];
    }
    denom[0] = (float)N;
    loss[0] = N > 0 ? (float)(L / (double)N) : 0.f;
  }
}

}  // namespace zs

extern "C" size_t zs_xent_forward_workspace(int64_t T, int64_t V) {
  const int64_t nparts = 2 * ((V + 255) / 256);
  return (size_t)(T * nparts * 2 + T) * sizeof(float) + 256;
}

extern "C" int zs_xent_forward(const void* hidden, int64_t T, int64_t D, int64_t h_sm, const void* classifier,
                               int64_t V, int64_t c_sm, const int64_t* labels, int s_max, const int* s_count,
                               float* lse, float* row_loss, float* loss, float* denom, void* workspace,
                               size_t workspace_bytes, int dtype, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ZS_REQUIRE(hidden && classifier && labels && s_count && lse && row_loss && loss && denom, ZS_ERR_ARG);
  ZS_REQUIRE(dtype == ZS_BF16 || dtype == ZS_F16, ZS_ERR_DTYPE);
  ZS_REQUIRE(T >= 1 && D >= 1 && V >= 1 && s_max >= 1 && s_max <= 8, ZS_ERR_SHAPE);
  ZS_REQUIRE(T < ((int64_t)1 << 31) && V < ((int64_t)1 << 31) && D < ((int64_t)1 << 24), ZS_ERR_SHAPE);
  ZS_REQUIRE(workspace && workspace_bytes >= zs_xent_forward_workspace(T, V), ZS_ERR_WORKSPACE);
  ZS_BIND(hidden);
  const int es = elem_size(dtype);
  constexpr int BN = 256;
  const int64_t n_vt = (V + BN - 1) / BN;
  float* ws = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  float* part_max = ws;
  float* part_sum = ws + T * 2 * n_vt;
  float* target_sum = part_sum + T * 2 * n_vt;
  ZS_CUDA_TRY(cudaMemsetAsync(target_sum, 0, sizeof(float) * T, stream));
  CUtensorMap tmA, tmB;
  int rc = make_tmap(&tmA, hidden, dtype, (uint64_t)D, (uint64_t)T, (uint64_t)h_sm * es, 64, 128);
  if (rc != ZS_OK) return rc;
  rc = make_tmap(&tmB, classifier, dtype, (uint64_t)D, (uint64_t)V, (uint64_t)c_sm * es, 64, BN / 2);
  if (rc != ZS_OK) return rc;
  GemmArgs a{};
  a.mode = MODE_ROWS;
  a.num_experts = 1;
  a.n_tiles = (int)n_vt;
  a.kb_rows = (int)((D + BK - 1) / BK);
  a.N_out = (int)V;
  a.n_rows = T;
  a.out_rows = T;
  a.out_dtype = dtype;
  a.b_rows_per_expert = 0;
  a.labels = labels;
  a.s_count = s_count;
  a.s_max = s_max;
  a.col_offset = 0;
  a.part_max = part_max;
  a.part_sum = part_sum;
  a.part_ld = 2 * n_vt;
  a.target_sum = target_sum;
  rc = launch_gemm<BN, 4, false, false, EPI_LSE>(tmA, tmB, a, ((T + BM - 1) / BM) * n_vt, stream);
  if (rc != ZS_OK) return rc;
  int64_t blocks = (T + 7) / 8;
  if (blocks > 148 * 16) blocks = 148 * 16;
  xent_finalize_kernel<<<(unsigned)blocks, 256, 0, stream>>>(part_max, part_sum, 2 * n_vt, (int)(2 * n_vt), target_sum,
                                                            s_count, s_max, T, lse, row_loss);
  ZS_CUDA_TRY(cudaGetLastError());
  xent_reduce_kernel<<<1, 1024, 0, stream>>>(row_loss, s_count, s_max, T, loss, denom);
  ZS_CUDA_TRY(cudaGetLastError());
  return ZS_OK;
}

extern "C" size_t zs_xent_backward_workspace(int64_t T, int64_t v_chunk, int dtype) {
  const int64_t pitch = ((v_chunk * elem_size(dtype) + 15) / 16) * 16;
  return (size_t)(T * pitch + 512);
}

namespace zs {
__global__ void xent_grad_scale_kernel(const float* __restrict__ grad_loss, const float* __restrict__ denom,
                                       float* __restrict__ out) {
  const float n = __ldg(denom);
  out[0] = n > 0.f ? __ldg(grad_loss) / n : 0.f;
}
}  // namespace zs

extern "C" int zs_xent_backward(const void* hidden, int64_t T, int64_t D, int64_t h_sm, const void* classifier,
                                int64_t V, int64_t c_sm, const int64_t* labels, int s_max, const int* s_count,
                                const float* lse, const float* grad_loss, const float* denom, float* d_hidden,
                                float* d_classifier, int64_t v_chunk, void* workspace, size_t workspace_bytes,
                                int dtype, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ZS_REQUIRE(hidden && classifier && labels && s_count && lse && grad_loss && denom, ZS_ERR_ARG);
  ZS_REQUIRE(d_hidden || d_classifier, ZS_ERR_ARG);
  ZS_REQUIRE(dtype == ZS_BF16 || dtype == ZS_F16, ZS_ERR_DTYPE);
  ZS_REQUIRE(T >= 1 && D >= 1 && V >= 1 && s_max >= 1 && s_max <= 8, ZS_ERR_SHAPE);
  ZS_REQUIRE(T < ((int64_t)1 << 31) && V < ((int64_t)1 << 31) && D < ((int64_t)1 << 24), ZS_ERR_SHAPE);
  ZS_REQUIRE(v_chunk >= 256 && v_chunk % 256 == 0, ZS_ERR_SHAPE);
  ZS_REQUIRE(workspace && workspace_bytes >= zs_xent_backward_workspace(T, v_chunk, dtype), ZS_ERR_WORKSPACE);
  ZS_REQUIRE((D * 4) % 16 == 0, ZS_ERR_ALIGN);
  ZS_BIND(hidden);
  const int es = elem_size(dtype);
  constexpr int BN = 256;
  const int64_t pitch = ((v_chunk * es + 15) / 16) * 16 / es;
  char* G = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  float* gscale = reinterpret_cast<float*>(G + ((T * pitch * es + 255) / 256) * 256);   // grad_loss / N
  xent_grad_scale_kernel<<<1, 1, 0, stream>>>(grad_loss, denom, gscale);
  ZS_CUDA_TRY(cudaGetLastError());
  CUtensorMap tmH_k, tmC_k, tmC_mn, tmH_mn;
  int rc = make_tmap(&tmH_k, hidden, dtype, (uint64_t)D, (uint64_t)T, (uint64_t)h_sm * es, 64, 128);
  if (rc != ZS_OK) return rc;
  rc = make_tmap(&tmC_k, classifier, dtype, (uint64_t)D, (uint64_t)V, (uint64_t)c_sm * es, 64, BN / 2);
  if (rc != ZS_OK) return rc;
  rc = make_tmap(&tmC_mn, classifier, dtype, (uint64_t)D, (uint64_t)V, (uint64_t)c_sm * es, 64, 64);
  if (rc != ZS_OK) return rc;
  rc = make_tmap(&tmH_mn, hidden, dtype, (uint64_t)D, (uint64_t)T, (uint64_t)h_sm * es, 64, 64);
  if (rc != ZS_OK) return rc;
  for (int64_t v0 = 0; v0 < V; v0 += v_chunk) {
    const int64_t vc = (V - v0 < v_chunk) ? (V - v0) : v_chunk;
    // (1) recompute the logits of this vocabulary slice; epilogue writes the
    //     logit gradient G = scale * (s * softmax - counts) in the input dtype
    GemmArgs g{};
    g.mode = MODE_ROWS;
    g.num_experts = 1;
    g.n_tiles = (int)((vc + BN - 1) / BN);
    g.kb_rows = (int)((D + BK - 1) / BK);
    g.N_out = (int)vc;
    g.n_rows = T;
    g.out_rows = T;
    g.out_dtype = dtype;
    g.out = G;
    g.ldo_m = pitch;
    g.ldo_n = 1;
    g.vec_ok = (pitch * es) % 16 == 0;
    g.b_row_offset = v0;
    g.labels = labels;
    g.s_count = s_count;
    g.s_max = s_max;
    g.col_offset = v0;
    g.lse = lse;
    g.grad_loss = grad_loss;
    g.denom = denom;
    rc = launch_gemm<BN, 4, false, false, EPI_XENT_GRAD>(tmH_k, tmC_k, g, ((T + BM - 1) / BM) * g.n_tiles, stream);
    if (rc != ZS_OK) return rc;
    CUtensorMap tmG_k, tmG_mn;
    rc = make_tmap(&tmG_k, G, dtype, (uint64_t)vc, (uint64_t)T, (uint64_t)pitch * es, 64, 128);
    if (rc != ZS_OK) return rc;
    rc = make_tmap(&tmG_mn, G, dtype, (uint64_t)vc, (uint64_t)T, (uint64_t)pitch * es, 64, 64);
    if (rc != ZS_OK) return rc;
    // (2) d_hidden (+)= G @ classifier[v0:v0+vc]
    if (d_hidden) {
      GemmArgs h{};
      h.mode = MODE_ROWS;
      h.num_experts = 1;
      h.n_tiles = (int)((D + BN - 1) / BN);
      h.kb_rows = (int)((vc + BK - 1) / BK);
      h.N_out = (int)D;
      h.n_rows = T;
      h.out_rows = T;
      h.out_dtype = dtype;
      h.out = reinterpret_cast<char*>(d_hidden);
      h.ldo_m = D;
      h.ldo_n = 1;
      h.vec_ok = (reinterpret_cast<uintptr_t>(d_hidden) % 16) == 0;
      h.b_row_offset = v0;
      h.accumulate = v0 > 0;
      h.f32_scale = gscale;
      rc = launch_gemm<BN, 4, false, true, EPI_F32>(tmG_k, tmC_mn, h, ((T + BM - 1) / BM) * h.n_tiles, stream);
      if (rc != ZS_OK) return rc;
    }
    // (3) d_classifier[v0:v0+vc] = G^T @ hidden
    if (d_classifier) {
      GemmArgs w{};
      w.mode = MODE_XTY;
      w.num_experts = 1;
      w.n_tiles = (int)((D + BN - 1) / BN);
      w.m_tiles_xty = (int)((vc + BM - 1) / BM);
      w.M_xty = (int)vc;
      w.N_out = (int)D;
      w.n_rows = T;
      w.out_dtype = dtype;
      w.out = reinterpret_cast<char*>(d_classifier + v0 * D);
      w.ldo_m = D;
      w.ldo_n = 1;
      w.out_se = 0;
      w.vec_ok = (reinterpret_cast<uintptr_t>(d_classifier) % 16) == 0;
      w.accumulate = 0;
      w.f32_scale = gscale;
      rc = launch_gemm<BN, 4, true, true, EPI_F32>(tmG_mn, tmH_mn, w, (int64_t)w.m_tiles_xty * w.n_tiles, stream);
      if (rc != ZS_OK) return rc;
    }
  }
  return ZS_OK;
}


// ------------------------------------------------------------ Newton-Schulz

namespace zs {
// Per-matrix Frobenius normalisation in the storage dtype, as
// X / (X.norm(dim=(-2,-1), keepdim=True) + 1e-7) evaluates it on a bf16 tensor:
// the norm (f32 accumulation) is rounded to the dtype, the sum with 1e-7 and
// the quotient each round once more.
// Deterministic two-level reduction over 16-byte vectors: NS_SUMSQ_BLOCKS
// blocks per matrix write partial sums of squares (fixed split, no atomics),
// one thread per matrix adds them in order and forms the divisor, then a
// grid-wide pass divides.  The result does not depend on the batch size.
constexpr int NS_SUMSQ_BLOCKS = 32;

template <typename T>
__global__ void ns_sumsq_kernel(const T* __restrict__ x, float* __restrict__ partial, int64_t per_vec) {
  const int64_t e = blockIdx.y;
  const uint4* xe = reinterpret_cast<const uint4*>(x) + e * per_vec;
  float ss = 0.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < per_vec; i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 u = __ldg(xe + i);
    const T* t = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float v = to_f32<T>(t[k]);
      ss = fmaf(v, v, ss);
    }
  }
  __shared__ float sh[32];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.f;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (threadIdx.x == 0) partial[e * NS_SUMSQ_BLOCKS + blockIdx.x] = v;
  }
}

// the divisor as X / (X.norm() + 1e-7) forms it on a 16-bit tensor: the norm
// (f32 accumulation) rounds to the dtype, so do the sum with 1e-7
template <typename T>
__global__ void ns_divisor_kernel(float* __restrict__ partial, int64_t batch) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= batch) return;
  float ss = 0.f;
  for (int b = 0; b < NS_SUMSQ_BLOCKS; ++b) ss += partial[e * NS_SUMSQ_BLOCKS + b];
  const float nrm = to_f32<T>(from_f32<T>(sqrtf(ss)));
  partial[e * NS_SUMSQ_BLOCKS] = to_f32<T>(from_f32<T>(nrm + 1e-7f));
}

template <typename T>
__global__ void ns_scale_kernel(const T* __restrict__ x, T* __restrict__ y, const float* __restrict__ div,
                                int64_t per_vec, int64_t total_vec) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total_vec;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = i / per_vec;
    const float den = __ldg(div + e * NS_SUMSQ_BLOCKS);
    uint4 u = __ldg(reinterpret_cast<const uint4*>(x) + i);
    T* t = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int k = 0; k < 8; ++k) t[k] = from_f32<T>(__fdiv_rn(to_f32<T>(t[k]), den));
    reinterpret_cast<uint4*>(y)[i] = u;
  }
}

template <typename T>
static int ns_normalize(const void* G, void* X, float* partial, int64_t batch, int64_t per, cudaStream_t stream) {
  const int64_t per_vec = per / 8;
  ns_sumsq_kernel<T><<<dim3((unsigned)NS_SUMSQ_BLOCKS, (unsigned)batch), 256, 0, stream>>>(
      reinterpret_cast<const T*>(G), partial, per_vec);
  ZS_CUDA_TRY(cudaGetLastError());
  ns_divisor_kernel<T><<<(unsigned)((batch + 127) / 128), 128, 0, stream>>>(partial, batch);
  ZS_CUDA_TRY(cudaGetLastError());
  const int64_t total = batch * per_vec;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  ns_scale_kernel<T><<<(unsigned)blocks, 256, 0, stream>>>(reinterpret_cast<const T*>(G), reinterpret_cast<T*>(X),
                                                           partial, per_vec, total);
  ZS_CUDA_TRY(cudaGetLastError());
  return ZS_OK;
}
}  // namespace zs

extern "C" size_t zs_newton_schulz5_workspace(int64_t batch, int64_t m, int64_t n, int dtype) {
  const int es = elem_size(dtype);
  return (size_t)(2 * batch * m * m + batch * m * n) * es + (size_t)((batch * 32 * 4 + 255) / 256) * 256 + 4 * 256;
}

extern "C" int zs_newton_schulz5(const void* G, void* X_out, int64_t batch, int64_t m, int64_t n, int steps, float a,
                                 float b, float c, void* workspace, size_t workspace_bytes, int dtype, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ZS_REQUIRE(G && X_out, ZS_ERR_ARG);
  ZS_REQUIRE(dtype == ZS_BF16 || dtype == ZS_F16, ZS_ERR_DTYPE);
  ZS_REQUIRE(batch >= 1 && m >= 1 && n >= m && steps >= 0, ZS_ERR_SHAPE);
  ZS_REQUIRE(batch * m < ((int64_t)1 << 31) && batch <= MAX_EXPERTS_GEMM && n < ((int64_t)1 << 24), ZS_ERR_SHAPE);
  ZS_REQUIRE((m * elem_size(dtype)) % 16 == 0 && (n * elem_size(dtype)) % 16 == 0, ZS_ERR_ALIGN);
  ZS_REQUIRE(workspace && workspace_bytes >= zs_newton_schulz5_workspace(batch, m, n, dtype), ZS_ERR_WORKSPACE);
  ZS_REQUIRE((reinterpret_cast<uintptr_t>(G) % 16) == 0 && (reinterpret_cast<uintptr_t>(X_out) % 16) == 0,
             ZS_ERR_ALIGN);
  ZS_BIND(G);
  const int es = elem_size(dtype);
  constexpr int BN = 256;
  char* ws = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  char* Abuf = ws;
  char* Bbuf = Abuf + ((batch * m * m * es + 255) / 256) * 256;
  char* Xtmp = Bbuf + ((batch * m * m * es + 255) / 256) * 256;
  float* ss = reinterpret_cast<float*>(Xtmp + ((batch * m * n * es + 255) / 256) * 256);  // [batch, 32] partials
  // X0 = G / (||G|| + 1e-7); the iterates alternate between two buffers, X0 placed so
  // that the last one lands in X_out (no final copy)
  char* X = (steps & 1) ? Xtmp : reinterpret_cast<char*>(X_out);
  char* Xn = (steps & 1) ? reinterpret_cast<char*>(X_out) : Xtmp;
  {
    const int rc = dtype == ZS_BF16 ? ns_normalize<__nv_bfloat16>(G, X, ss, batch, m * n, stream)
                                    : ns_normalize<__half>(G, X, ss, batch, m * n, stream);
    if (rc != ZS_OK) return rc;
  }
  for (int it = 0; it < steps; ++it) {
    CUtensorMap tX_k128, tX_k256, tX_mn, tA_k128, tA_k256, tB_k128, tO_A, tO_B, tO_X, tA_mn, tB_mn;
    int rc;
    // A and B are symmetric: with pair tiles only their upper 256 x 256 tiles are written,
    // and the products that read them take the blocks left of the diagonal transposed
    if ((rc = make_tmap(&tA_mn, Abuf, dtype, m, batch * m, m * es, 64, 64)) != ZS_OK) return rc;
    if ((rc = make_tmap(&tB_mn, Bbuf, dtype, m, batch * m, m * es, 64, 64)) != ZS_OK) return rc;
    // outputs of the three products, written by TMA stores
    if ((rc = make_out_tmap(&tO_A, Abuf, dtype, m, batch * m, m * es)) != ZS_OK) return rc;
    if ((rc = make_out_tmap(&tO_B, Bbuf, dtype, m, batch * m, m * es)) != ZS_OK) return rc;
    if ((rc = make_out_tmap(&tO_X, Xn, dtype, n, batch * m, n * es)) != ZS_OK) return rc;
    if ((rc = make_tmap(&tX_k128, X, dtype, n, batch * m, n * es, 64, 128)) != ZS_OK) return rc;
    if ((rc = make_tmap(&tX_k256, X, dtype, n, batch * m, n * es, 64, BN / 2)) != ZS_OK) return rc;
    if ((rc = make_tmap(&tX_mn, X, dtype, n, batch * m, n * es, 64, 64)) != ZS_OK) return rc;
    if ((rc = make_tmap(&tA_k128, Abuf, dtype, m, batch * m, m * es, 64, 128)) != ZS_OK) return rc;
    if ((rc = make_tmap(&tA_k256, Abuf, dtype, m, batch * m, m * es, 64, BN / 2)) != ZS_OK) return rc;
    if ((rc = make_tmap(&tB_k128, Bbuf, dtype, m, batch * m, m * es, 64, 128)) != ZS_OK) return rc;
    GemmArgs g{};
    g.mode = MODE_ROWS;
    g.num_experts = (int)batch;
    g.group_rows = m;
    g.n_rows = batch * m;
    g.out_rows = batch * m;
    g.out_dtype = dtype;
    g.ldo_n = 1;
    g.tma_store = 1;
    const int64_t mt = (m + BM - 1) / BM;
    // A = X X^T  (per matrix: M = m, N = m, K = n; B operand = X rows of the same matrix)
    g.n_tiles = (int)((m + BN - 1) / BN);
    g.kb_rows = (int)((n + BK - 1) / BK);
    g.N_out = (int)m;
    g.out = Abuf;
    g.ldo_m = m;
    g.b_rows_per_expert = (int)m;
    g.vec_ok = 1;
    // X X^T and A A are symmetric: on 256 x 256 pair tiles only the upper
    // triangle of tiles is computed, each off-diagonal tile also writes its
    // transpose (the third product, B X, is not symmetric)
    g.sym_upper = (pair_enabled() && m % 256 == 0) ? 1 : 0;
    const int sym = g.sym_upper && sym_operands_enabled();
    g.sym_ops = sym ? 4 : 0;   // output only: neither operand is symmetric, the mirror is skipped
    if ((rc = launch_gemm<BN, 4, false, false, EPI_STORE>(tX_k128, tX_k256, g, batch * mt * g.n_tiles, stream,
                                                          &tO_A)) != ZS_OK)
      return rc;
    // B = b A + c A A   (B operand = A^T = A)
    g.kb_rows = (int)((m + BK - 1) / BK);
    g.out = Bbuf;
    g.aux = Abuf;
    g.ld_aux = m;
    g.alpha = c;
    g.beta = b;
    g.sym_ops = sym ? 3 : 0;   // both operands are A (upper tiles stored)
    if ((rc = launch_gemm<BN, 4, false, false, EPI_AXPBY>(tA_k128, tA_k256, g, batch * mt * g.n_tiles, stream,
                                                          &tO_B, &tA_mn, &tA_mn)) != ZS_OK)
      return rc;
    // X' = a X + B X    (B operand = X^T: X is [K = m rows, N = n cols] per matrix, MN-major)
    g.sym_upper = 0;
    g.n_tiles = (int)((n + BN - 1) / BN);
    g.kb_rows = (int)((m + BK - 1) / BK);
    g.N_out = (int)n;
    g.out = Xn;
    g.ldo_m = n;
    g.aux = X;
    g.ld_aux = n;
    g.alpha = 1.0f;
    g.beta = a;
    g.b_rows_per_expert = (int)m;
    g.sym_ops = sym ? 1 : 0;   // A = B (upper tiles stored); X is whole
    if ((rc = launch_gemm<BN, 4, false, true, EPI_AXPBY>(tB_k128, tX_mn, g, batch * mt * g.n_tiles, stream,
                                                         &tO_X, &tB_mn)) != ZS_OK)
      return rc;
    char* t = X;
    X = Xn;
    Xn = t;
  }
  return ZS_OK;
}
