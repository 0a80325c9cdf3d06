// The sparse input embedding of the training step: the bag-mean lookup with the
// sqrt(d) upscale (modeling/model.py:71-86 of the reference) as one gather pass,
// its gradient in the COO form nn.Embedding(sparse=True) produces, and the
// per-row RMSProp + unit-sphere step on that gradient
// (engram/GramReaperSparse.py:18-66) as device kernels without host syncs.
//
// The optimizer step is a stable LSD radix sort of the lookups by table row
// (8-bit digits: per-chunk histograms, one scan block, a stable scatter), then
// one CTA per distinct row: the row's gradient is summed over its lookups in
// their original order (deterministic, the coalesce of the reference), and the
// RMSProp update, the renormalisation and the store run on registers.
#include "zs_common.cuh"

namespace zs {

// ------------------------------------------------------------ embedding bag --

// out[t, :] = scale * mean_j table[ids[t, j], :]   (f32; j < bag, mean = sum * (1/bag))
// One warp per output row, 16-byte accesses (d % 4 == 0).
__global__ void embedding_bag_fwd_kernel(const float* __restrict__ table, int64_t num_rows, int64_t d,
                                         const int64_t* __restrict__ ids, int64_t T, int bag, float scale,
                                         float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t nv = d / 4;
  const float inv = 1.0f / (float)bag;
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T; t += warps) {
    float4* orow = reinterpret_cast<float4*>(out + t * d);
    for (int64_t v0 = 0; v0 < nv; v0 += 64) {
      float4 acc[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
      for (int j = 0; j < bag; ++j) {
        const int64_t r = __ldg(ids + t * bag + j);
        if (r < 0 || r >= num_rows) {
          if (lane == 0 && v0 == 0) record_error(ZS_DEVERR_INDEX);
          continue;
        }
        const float4* src = reinterpret_cast<const float4*>(table + r * d);
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int64_t v = v0 + u * 32 + lane;
          if (v < nv) {
            const float4 a = __ldg(src + v);
            acc[u].x += a.x; acc[u].y += a.y; acc[u].z += a.z; acc[u].w += a.w;
          }
        }
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int64_t v = v0 + u * 32 + lane;
        if (v >= nv) continue;
        float4 o = acc[u];
        if (bag > 1) {
          // the reference's bag.float().mean(-2): the f32 sum times 1/bag
          o.x *= inv; o.y *= inv; o.z *= inv; o.w *= inv;
        }
        o.x *= scale; o.y *= scale; o.z *= scale; o.w *= scale;
        orow[v] = o;
      }
    }
  }
}

// values[t * bag + j, :] = (dy[t, :] * scale) / bag   (the COO values of the lookups)
__global__ void embedding_bag_bwd_kernel(const float* __restrict__ dy, int64_t T, int bag, int64_t d, float scale,
                                         float* __restrict__ values) {
  const int64_t nv = d / 4;
  const int64_t total = T * nv;
  const float fb = (float)bag;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / nv, v = i - t * nv;
    float4 g = __ldg(reinterpret_cast<const float4*>(dy) + i);
    g.x *= scale; g.y *= scale; g.z *= scale; g.w *= scale;
    if (bag > 1) {
      g.x /= fb; g.y /= fb; g.z /= fb; g.w /= fb;
    }
    for (int j = 0; j < bag; ++j) reinterpret_cast<float4*>(values + (t * bag + j) * d)[v] = g;
  }
}

// -------------------------------------------------------- row radix sort --

constexpr int RS_CHUNK = 4096;   // lookups per block of a pass
constexpr int RS_THREADS = 256;
constexpr int RS_BINS = 256;     // 8-bit digits

__device__ __forceinline__ int rs_key(const int64_t* rows, const int* perm, int64_t i, int64_t num_rows) {
  const int64_t r = rows[perm ? perm[i] : i];
  return (r < 0 || r >= num_rows) ? (int)num_rows : (int)r;   // out-of-range rows sort last (sentinel)
}

__global__ void rs_hist_kernel(const int64_t* __restrict__ rows, const int* __restrict__ perm, int64_t n,
                               int64_t num_rows, int shift, int* __restrict__ hist) {
  __shared__ int sh[RS_BINS];
  for (int b = threadIdx.x; b < RS_BINS; b += blockDim.x) sh[b] = 0;
  __syncthreads();
  const int64_t beg = (int64_t)blockIdx.x * RS_CHUNK, end = min(beg + RS_CHUNK, n);
  for (int64_t i = beg + threadIdx.x; i < end; i += blockDim.x)
    atomicAdd(&sh[(rs_key(rows, perm, i, num_rows) >> shift) & (RS_BINS - 1)], 1);
  __syncthreads();
  for (int b = threadIdx.x; b < RS_BINS; b += blockDim.x) hist[(int64_t)blockIdx.x * RS_BINS + b] = sh[b];
}

// One block: hist[blk][b] -> global start of digit b's slice for chunk blk.
__global__ void rs_scan_kernel(int* __restrict__ hist, int nblk) {
  __shared__ int tot[RS_BINS];
  for (int b = threadIdx.x; b < RS_BINS; b += blockDim.x) {
    int run = 0;
    for (int blk = 0; blk < nblk; ++blk) {
      const int c = hist[blk * RS_BINS + b];
      hist[blk * RS_BINS + b] = run;
      run += c;
    }
    tot[b] = run;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int b = 0; b < RS_BINS; ++b) {
      const int c = tot[b];
      tot[b] = run;
      run += c;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < nblk * RS_BINS; i += blockDim.x) hist[i] += tot[i % RS_BINS];
}

// Stable scatter of one digit pass: within a step of 256 lookups the rank of a
// lookup among equal digits is the digit's running count + equal digits in lower
// warps + equal digits in lower lanes.
__global__ void rs_scatter_kernel(const int64_t* __restrict__ rows, const int* __restrict__ perm_in, int64_t n,
                                  int64_t num_rows, int shift, const int* __restrict__ hist, int* __restrict__ perm_out) {
  constexpr int W = RS_THREADS / 32;
  __shared__ int running[RS_BINS];
  __shared__ int wcnt[W][RS_BINS];
  for (int b = threadIdx.x; b < RS_BINS; b += blockDim.x) running[b] = hist[(int64_t)blockIdx.x * RS_BINS + b];
  for (int x = threadIdx.x; x < W * RS_BINS; x += blockDim.x) (&wcnt[0][0])[x] = 0;
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t lt = (1u << lane) - 1u;
  const int64_t beg = (int64_t)blockIdx.x * RS_CHUNK, end = min(beg + RS_CHUNK, n);
  for (int64_t s = beg; s < end; s += RS_THREADS) {
    const int64_t i = s + threadIdx.x;
    int dg = -1, src = 0;
    if (i < end) {
      src = perm_in ? perm_in[i] : (int)i;
      dg = (rs_key(rows, perm_in, i, num_rows) >> shift) & (RS_BINS - 1);
    }
    const uint32_t peers = __match_any_sync(0xffffffffu, dg);
    const int rank = __popc(peers & lt);
    const int cnt = __popc(peers);
    if (dg >= 0 && rank == 0) wcnt[warp][dg] = cnt;
    __syncthreads();
    int pos = 0;
    if (dg >= 0) {
      pos = running[dg] + rank;
      for (int w = 0; w < warp; ++w) pos += wcnt[w][dg];
    }
    __syncthreads();
    if (dg >= 0) {
      perm_out[pos] = src;
      if (rank == 0) {
        atomicAdd(&running[dg], cnt);
        wcnt[warp][dg] = 0;
      }
    }
    __syncthreads();
  }
}

// ------------------------------------------------------- per-row RMSProp --

__global__ void rs_tick_kernel(long long* __restrict__ step) { *step += 1; }

constexpr int RMS_THREADS = 128;
constexpr int RMS_ITEMS = 8;   // float4 per thread: d <= 128 * 8 * 4 = 4096

__device__ __forceinline__ float rms_block_sum(float v, float* red) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < RMS_THREADS / 32; ++w) s += red[w];
  return s;
}

// One CTA per sorted position; the CTA at the first lookup of a row owns the row:
//   g   = sum of the row's lookup gradients (in lookup order)
//   v   = beta * v + (1 - beta) * sum(g^2)
//   p  -= lr / (sqrt(v / (1 - beta^t)) + eps) * g
//   p  /= max(||p||, eps)            (unit_norm)
__global__ void __launch_bounds__(RMS_THREADS) rs_rmsprop_kernel(
    const int64_t* __restrict__ rows, const int* __restrict__ perm, int64_t n, int64_t num_rows,
    const float* __restrict__ values, int64_t ld_val, float* __restrict__ p, int64_t ld_p, int64_t d,
    float* __restrict__ v_state, const long long* __restrict__ step, const float* __restrict__ lr_ptr, float lr_val,
    double beta, float eps, int unit_norm) {
  __shared__ float red[RMS_THREADS / 32];
  const int64_t i = blockIdx.x;
  if (i >= n) return;
  const int64_t r = rs_key(rows, perm, i, num_rows);
  if (r >= num_rows) {
    if (threadIdx.x == 0 && (i == 0 || rs_key(rows, perm, i - 1, num_rows) != r)) record_error(ZS_DEVERR_INDEX);
    return;
  }
  if (i > 0 && rs_key(rows, perm, i - 1, num_rows) == r) return;   // not the first lookup of the row
  const int64_t nv = d / 4;
  float4 g[RMS_ITEMS];
#pragma unroll
  for (int u = 0; u < RMS_ITEMS; ++u) g[u] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int64_t j = i; j < n && rs_key(rows, perm, j, num_rows) == r; ++j) {
    const float4* src = reinterpret_cast<const float4*>(values + (int64_t)perm[j] * ld_val);
#pragma unroll
    for (int u = 0; u < RMS_ITEMS; ++u) {
      const int64_t v = u * RMS_THREADS + threadIdx.x;
      if (v < nv) {
        const float4 a = __ldg(src + v);
        g[u].x += a.x; g[u].y += a.y; g[u].z += a.z; g[u].w += a.w;
      }
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int u = 0; u < RMS_ITEMS; ++u)
    ss += g[u].x * g[u].x + g[u].y * g[u].y + g[u].z * g[u].z + g[u].w * g[u].w;
  ss = rms_block_sum(ss, red);
  const float b = (float)beta;
  const float one_minus_b = (float)(1.0 - beta);
  const float vn = b * v_state[r] + one_minus_b * ss;
  const float bc = (float)(1.0 - pow(beta, (double)*step));
  const float lr = lr_ptr ? *lr_ptr : lr_val;
  const float stepsize = lr / (sqrtf(vn / bc) + eps);
  float4* prow = reinterpret_cast<float4*>(p + r * ld_p);
  float4 w[RMS_ITEMS];
  float nn = 0.f;
#pragma unroll
  for (int u = 0; u < RMS_ITEMS; ++u) {
    const int64_t v = u * RMS_THREADS + threadIdx.x;
    w[u] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (v < nv) {
      const float4 a = prow[v];
      w[u] = make_float4(a.x - stepsize * g[u].x, a.y - stepsize * g[u].y, a.z - stepsize * g[u].z,
                         a.w - stepsize * g[u].w);
      nn += w[u].x * w[u].x + w[u].y * w[u].y + w[u].z * w[u].z + w[u].w * w[u].w;
    }
  }
  float den = 1.f;
  if (unit_norm) den = fmaxf(sqrtf(rms_block_sum(nn, red)), eps);
#pragma unroll
  for (int u = 0; u < RMS_ITEMS; ++u) {
    const int64_t v = u * RMS_THREADS + threadIdx.x;
    if (v < nv) {
      float4 o = w[u];
      if (unit_norm) {
        o.x /= den; o.y /= den; o.z /= den; o.w /= den;
      }
      prow[v] = o;
    }
  }
  if (threadIdx.x == 0) v_state[r] = vn;
}

static int rs_passes(int64_t num_rows) {
  int bits = 0;
  while (((int64_t)1 << bits) <= num_rows) ++bits;   // the sentinel num_rows must fit too
  return (bits + 7) / 8;
}

}  // namespace zs

using namespace zs;

extern "C" int zs_embedding_bag_forward(const float* table, int64_t num_rows, int64_t d, const int64_t* ids,
                                        int64_t num_bags, int bag, float scale, float* out, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ZS_REQUIRE(table && out && (num_bags == 0 || ids), ZS_ERR_ARG);
  ZS_REQUIRE(num_rows >= 1 && d >= 4 && d % 4 == 0 && bag >= 1 && num_bags >= 0, ZS_ERR_SHAPE);
  ZS_REQUIRE(((reinterpret_cast<uintptr_t>(table) | reinterpret_cast<uintptr_t>(out)) % 16) == 0, ZS_ERR_ALIGN);
  ZS_BIND(table);
  if (num_bags == 0) return ZS_OK;
  int64_t blocks = (num_bags + 7) / 8;
  if (blocks > 148 * 16) blocks = 148 * 16;
  embedding_bag_fwd_kernel<<<(unsigned)blocks, 256, 0, stream>>>(table, num_rows, d, ids, num_bags, bag, scale, out);
  ZS_CUDA_TRY(cudaGetLastError());
  return ZS_OK;
}

extern "C" int zs_embedding_bag_backward(const float* dy, int64_t num_bags, int bag, int64_t d, float scale,
                                         float* values, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ZS_REQUIRE(num_bags == 0 || (dy && values), ZS_ERR_ARG);
  ZS_REQUIRE(d >= 4 && d % 4 == 0 && bag >= 1 && num_bags >= 0, ZS_ERR_SHAPE);
  ZS_REQUIRE(((reinterpret_cast<uintptr_t>(dy) | reinterpret_cast<uintptr_t>(values)) % 16) == 0, ZS_ERR_ALIGN);
  if (num_bags == 0) return ZS_OK;
  ZS_BIND(dy);
  const int64_t total = num_bags * (d / 4);
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  embedding_bag_bwd_kernel<<<(unsigned)blocks, 256, 0, stream>>>(dy, num_bags, bag, d, scale, values);
  ZS_CUDA_TRY(cudaGetLastError());
  return ZS_OK;
}

extern "C" size_t zs_sparse_rmsprop_workspace(int64_t n, int64_t num_rows) {
  (void)num_rows;
  const int64_t nblk = (n + RS_CHUNK - 1) / RS_CHUNK;
  return (size_t)(2 * ((n + 63) / 64) * 64 + (nblk > 0 ? nblk : 1) * RS_BINS) * sizeof(int) + 256;
}

extern "C" int zs_sparse_rmsprop_step(float* param, int64_t num_rows, int64_t d, int64_t ld_param, float* v_state,
                                      long long* step_counter, const int64_t* rows, const float* values,
                                      int64_t ld_values, int64_t n, const float* lr_ptr, float lr, double beta,
                                      float eps, int unit_norm, void* workspace, size_t workspace_bytes,
                                      void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ZS_REQUIRE(param && v_state && step_counter, ZS_ERR_ARG);
  ZS_REQUIRE(n == 0 || (rows && values), ZS_ERR_ARG);
  ZS_REQUIRE(num_rows >= 1 && num_rows < ((int64_t)1 << 31) - 1 && n >= 0 && n < ((int64_t)1 << 31), ZS_ERR_SHAPE);
  ZS_REQUIRE(d >= 4 && d % 4 == 0 && d <= (int64_t)RMS_THREADS * RMS_ITEMS * 4, ZS_ERR_SHAPE);
  ZS_REQUIRE(ld_param >= d && ld_param % 4 == 0 && ld_values >= d && ld_values % 4 == 0, ZS_ERR_SHAPE);
  ZS_REQUIRE(((reinterpret_cast<uintptr_t>(param) | reinterpret_cast<uintptr_t>(values)) % 16) == 0, ZS_ERR_ALIGN);
  ZS_BIND(param);
  if (n == 0) return ZS_OK;   // nothing touched: the step counter does not advance (as the reference skips)
  ZS_REQUIRE(workspace && workspace_bytes >= zs_sparse_rmsprop_workspace(n, num_rows), ZS_ERR_WORKSPACE);
  int* ws = reinterpret_cast<int*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  const int64_t npad = ((n + 63) / 64) * 64;
  int* perm[2] = {ws, ws + npad};
  int* hist = ws + 2 * npad;
  const int nblk = (int)((n + RS_CHUNK - 1) / RS_CHUNK);
  rs_tick_kernel<<<1, 1, 0, stream>>>(step_counter);
  ZS_CUDA_TRY(cudaGetLastError());
  const int passes = rs_passes(num_rows);
  const int* cur = nullptr;
  for (int ps = 0; ps < passes; ++ps) {
    rs_hist_kernel<<<nblk, RS_THREADS, 0, stream>>>(rows, cur, n, num_rows, 8 * ps, hist);
    ZS_CUDA_TRY(cudaGetLastError());
    rs_scan_kernel<<<1, RS_BINS, 0, stream>>>(hist, nblk);
    ZS_CUDA_TRY(cudaGetLastError());
    rs_scatter_kernel<<<nblk, RS_THREADS, 0, stream>>>(rows, cur, n, num_rows, 8 * ps, hist, perm[ps & 1]);
    ZS_CUDA_TRY(cudaGetLastError());
    cur = perm[ps & 1];
  }
  rs_rmsprop_kernel<<<(unsigned)n, RMS_THREADS, 0, stream>>>(rows, cur, n, num_rows, values, ld_values, param, ld_param,
                                                            d, v_state, step_counter, lr_ptr, lr, beta, eps, unit_norm);
  ZS_CUDA_TRY(cudaGetLastError());
  return ZS_OK;
}
