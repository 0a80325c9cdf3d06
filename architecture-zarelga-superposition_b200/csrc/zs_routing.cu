// Routing kernels of the MoE layer:
//   * gate_topk: MoEGate's biased top-k selection + L1-normalised weights
//     (modeling/moe_gate.py:29-34), one warp per token, bit-exact indices.
//   * flatten_sort_count: stable counting sort of the flat expert ids
//     (scattermoe/parallel_experts.py:21-28) in three launches: per-chunk
//     histograms, one scan block, and a stable scatter that ranks equal ids
//     with warp match + cross-warp prefix sums.
//   * bincount / expert counts / sign bias update
//     (scattermoe/parallel_experts.py:6-15, main.py:161-175).
#include "zs_common.cuh"

#include <mutex>

namespace zs {

// Total order on f32 used by CUDA torch.topk's radix select: flip so that
// unsigned comparison matches float comparison; NaN sorts above everything.
__device__ __forceinline__ uint32_t ordered_key(float v) {
  const uint32_t x = __float_as_uint(v);
  if (v != v) return 0xffffffffu;
  return (x & 0x80000000u) ? ~x : (x | 0x80000000u);
}

template <typename T>
__device__ __forceinline__ float ld_f32(const T* p) {
  return to_f32<T>(*p);
}

// One warp per token.  Lane l holds experts e = j*32 + l for j < VPL.
template <typename T, int VPL>
__global__ void gate_topk_kernel(const T* __restrict__ probs, const float* __restrict__ bias, int64_t num_tokens,
                                 int E, int k, int64_t* __restrict__ idx_out, T* __restrict__ w_out) {
  const int lane = threadIdx.x & 31;
  const uint32_t lt_mask = (1u << lane) - 1u;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < num_tokens; t += warps) {
    const T* row = probs + t * E;
    uint32_t key[VPL];
    uint32_t valid = 0;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int e = j * 32 + lane;
      if (e < E) {
        key[j] = ordered_key(ld_f32(row + e) + bias[e]);
        valid |= 1u << j;
      } else {
        key[j] = 0;
      }
    }
    // k rounds of warp arg-max; ties go to the lowest expert index, which is
    // the set CUDA's gatherTopK keeps at the k-th value.
    uint32_t sel = 0;
    uint32_t kth = 0;
    for (int r = 0; r < k; ++r) {
      uint32_t bk = 0;
      int be = 0x7fffffff;  // "none"
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        // e grows with j, so a strict '>' keeps the lower index on ties.
        const bool cand = ((valid & ~sel) >> j) & 1u;
        if (cand && (be == 0x7fffffff || key[j] > bk)) {
          bk = key[j];
          be = j * 32 + lane;
        }
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const uint32_t ok = __shfl_xor_sync(0xffffffffu, bk, off);
        const int oe = __shfl_xor_sync(0xffffffffu, be, off);
        const bool take = (oe != 0x7fffffff) &&
                          (be == 0x7fffffff || ok > bk || (ok == bk && oe < be));
        if (take) {
          bk = ok;
          be = oe;
        }
      }
      if (be != 0x7fffffff && (be & 31) == lane) sel |= 1u << (be >> 5);
      kth = bk;
    }
    // Output order of torch.topk(sorted=False) on CUDA: values strictly above
    // the k-th value in index order, then the k-th-value ties in index order.
    uint32_t gbits = 0, qbits = 0;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      if ((sel >> j) & 1u) {
        if (key[j] > kth)
          gbits |= 1u << j;
        else
          qbits |= 1u << j;
      }
    }
    int n_g = 0;
#pragma unroll
    for (int j = 0; j < VPL; ++j) n_g += __popc(__ballot_sync(0xffffffffu, (gbits >> j) & 1u));
    int base_g = 0, base_q = n_g;
    float wsum = 0.f;
    float myw[VPL];
    int mypos[VPL];
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const uint32_t bg = __ballot_sync(0xffffffffu, (gbits >> j) & 1u);
      const uint32_t bq = __ballot_sync(0xffffffffu, (qbits >> j) & 1u);
      mypos[j] = -1;
      if ((gbits >> j) & 1u) mypos[j] = base_g + __popc(bg & lt_mask);
      if ((qbits >> j) & 1u) mypos[j] = base_q + __popc(bq & lt_mask);
      base_g += __popc(bg);
      base_q += __popc(bq);
      myw[j] = 0.f;
      if (mypos[j] >= 0) {
        myw[j] = ld_f32(row + j * 32 + lane);
        wsum += fabsf(myw[j]);
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, off);
    // F.normalize(p=1): the norm is produced in the tensor dtype, clamped at
    // eps, and the division rounds once more to the tensor dtype.
    float denom = to_f32<T>(from_f32<T>(wsum));
    const float eps = to_f32<T>(from_f32<T>(1e-12f));
    if (denom < eps) denom = eps;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      if (mypos[j] >= 0) {
        idx_out[t * k + mypos[j]] = j * 32 + lane;
        w_out[t * k + mypos[j]] = from_f32<T>(__fdiv_rn(myw[j], denom));
      }
    }
  }
}

template <typename T>
static int launch_gate_topk(const void* probs, const float* bias, int64_t Tn, int E, int k, int64_t* idx, void* w,
                            cudaStream_t stream) {
  const int threads = 256;
  int64_t blocks = (Tn + 7) / 8;
  if (blocks > 148 * 32) blocks = 148 * 32;
  if (blocks < 1) blocks = 1;
  const T* p = reinterpret_cast<const T*>(probs);
  T* wo = reinterpret_cast<T*>(w);
  const int vpl = (E + 31) / 32;
#define ZS_TOPK_CASE(V)                                                                                    \
  if (vpl <= V) {                                                                                          \
    gate_topk_kernel<T, V><<<(unsigned)blocks, threads, 0, stream>>>(p, bias, Tn, E, k, idx, wo);          \
    return cudaGetLastError() == cudaSuccess ? ZS_OK : ZS_ERR_CUDA;                                        \
  }
  ZS_TOPK_CASE(1)
  ZS_TOPK_CASE(2)
  ZS_TOPK_CASE(4)
  ZS_TOPK_CASE(8)
  ZS_TOPK_CASE(16)
  ZS_TOPK_CASE(32)
#undef ZS_TOPK_CASE
  return ZS_ERR_SHAPE;
}

// ------------------------------------------------------ flatten_sort_count --

constexpr int FSC_CHUNK = 4096;   // ids per block
constexpr int FSC_THREADS = 256;

// Phase A: per-chunk histogram over num_experts + 1 buckets (the extra bucket
// collects out-of-range ids so every output slot stays defined).
__global__ void fsc_hist_kernel(const int64_t* __restrict__ ids, int64_t n, int E, int* __restrict__ hist) {
  extern __shared__ int sh[];
  const int B = E + 1;
  for (int b = threadIdx.x; b < B; b += blockDim.x) sh[b] = 0;
  __syncthreads();
  const int64_t beg = (int64_t)blockIdx.x * FSC_CHUNK;
  const int64_t end = min(beg + FSC_CHUNK, n);
  bool bad = false;
  for (int64_t i = beg + threadIdx.x; i < end; i += blockDim.x) {
    int64_t e = ids[i];
    if (e < 0 || e >= E) {
      bad = true;
      e = E;
    }
    atomicAdd(&sh[e], 1);
  }
  if (bad) record_error(ZS_DEVERR_INDEX);
  __syncthreads();
  for (int b = threadIdx.x; b < B; b += blockDim.x) hist[(int64_t)blockIdx.x * B + b] = sh[b];
}

// Phase B (one block): turn hist[blk][b] into the global start of bucket b's
// slice for block blk, and write the inclusive expert offsets.  The histogram
// is staged in shared memory when it fits (coalesced load, no dependent
// global-memory chains).
__global__ void fsc_scan_kernel(int* __restrict__ hist, int nblk, int E, int64_t* __restrict__ offsets,
                                int staged) {
  extern __shared__ int sh[];  // totals[B] (+ staged hist[nblk][B])
  const int B = E + 1;
  int* h = staged ? sh + B : hist;
  if (staged) {
    for (int i = threadIdx.x; i < nblk * B; i += blockDim.x) h[i] = hist[i];
    __syncthreads();
  }
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    int run = 0;
    for (int blk = 0; blk < nblk; ++blk) {
      const int c = h[blk * B + b];
      h[blk * B + b] = run;
      run += c;
    }
    sh[b] = run;
  }
  __syncthreads();
  // exclusive scan of the bucket totals (one warp; B <= 4097)
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    const int per = (B + 31) / 32;
    const int beg = lane * per, end = min(beg + per, B);
    int local = 0;
    for (int b = beg; b < end; ++b) local += sh[b];
    int incl = local;
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += v;
    }
    int run = incl - local;
    for (int b = beg; b < end; ++b) {
      const int c = sh[b];
      sh[b] = run;
      run += c;
      if (b < E) offsets[b] = run;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < nblk * B; i += blockDim.x) hist[i] = h[i] + sh[i % B];
}

// Phase C: stable scatter.  Each block walks its chunk in order, 256 ids per
// step; the rank of an id among equal ids is (running count of the bucket) +
// (equal ids in lower warps of this step) + (equal ids in lower lanes).
__global__ void fsc_scatter_kernel(const int64_t* __restrict__ ids, int64_t n, int E, const int* __restrict__ hist,
                                   int64_t* __restrict__ sorted_e, int64_t* __restrict__ sorted_i) {
  extern __shared__ int sh[];
  const int B = E + 1;
  constexpr int W = FSC_THREADS / 32;
  int* running = sh;          // [B]
  int* wcnt = sh + B;         // [W][B]
  for (int b = threadIdx.x; b < B; b += blockDim.x) running[b] = hist[(int64_t)blockIdx.x * B + b];
  for (int x = threadIdx.x; x < W * B; x += blockDim.x) wcnt[x] = 0;
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t lt_mask = (1u << lane) - 1u;
  const int64_t beg = (int64_t)blockIdx.x * FSC_CHUNK;
  const int64_t end = min(beg + FSC_CHUNK, n);
  for (int64_t s = beg; s < end; s += FSC_THREADS) {
    const int64_t i = s + threadIdx.x;
    int e = -1;
    if (i < end) {
      int64_t v = ids[i];
      e = (v < 0 || v >= E) ? E : (int)v;
    }
    const uint32_t peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & lt_mask);
    const bool leader = rank == 0;
    const int cnt = __popc(peers);
    if (e >= 0 && leader) wcnt[warp * B + e] = cnt;
    __syncthreads();
    int pos = 0;
    if (e >= 0) {
      pos = running[e] + rank;
      for (int w = 0; w < warp; ++w) pos += wcnt[w * B + e];
    }
    __syncthreads();
    if (e >= 0) {
      sorted_e[pos] = e;
      sorted_i[pos] = i;
      if (leader) {
        atomicAdd(&running[e], cnt);
        wcnt[warp * B + e] = 0;
      }
    }
    __syncthreads();
  }
}

// --------------------------------------------------------------- counting --

__global__ void count_kernel(const int64_t* __restrict__ x, const uint8_t* __restrict__ valid, int64_t n, int per_row,
                             int minlength, int64_t* __restrict__ out) {
  extern __shared__ int sh[];
  for (int b = threadIdx.x; b < minlength; b += blockDim.x) sh[b] = 0;
  __syncthreads();
  bool bad = false;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    if (valid != nullptr && valid[i / per_row] == 0) continue;
    const int64_t v = x[i];
    if (v < 0 || v >= minlength) {
      bad = true;
      continue;
    }
    atomicAdd(&sh[v], 1);
  }
  if (bad) record_error(ZS_DEVERR_INDEX);
  __syncthreads();
  for (int b = threadIdx.x; b < minlength; b += blockDim.x)
    if (sh[b]) atomicAdd(reinterpret_cast<unsigned long long*>(out + b), (unsigned long long)sh[b]);
}

__global__ void bias_sign_update_kernel(const int64_t* __restrict__ counts, int E, float rate, float* __restrict__ bias) {
  __shared__ float s_sum;
  __shared__ long long s_tot;
  if (threadIdx.x == 0) {
    long long tot = 0;
    for (int e = 0; e < E; ++e) tot += counts[e];
    s_tot = tot;
    // float(count) sums exactly below 2^24; mean = sum / E in f32 as torch does.
    s_sum = (float)tot;
  }
  __syncthreads();
  if (s_tot == 0) return;
  // torch's CUDA mean reduction multiplies the f32 sum by the f32 factor 1/E.
  const float mean = s_sum * __fdiv_rn(1.0f, (float)E);
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const float err = mean - (float)counts[e];
    const float sgn = err > 0.f ? 1.f : (err < 0.f ? -1.f : 0.f);
    bias[e] = bias[e] + rate * sgn;
  }
}

}  // namespace zs

using namespace zs;

extern "C" int zs_moe_gate_topk(const void* gate_probs, int probs_dtype, const float* expert_biases,
                                int64_t num_tokens, int num_experts, int top_k, int64_t* topk_idx, void* topk_weight,
                                void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ZS_REQUIRE(gate_probs && expert_biases && topk_idx && topk_weight, ZS_ERR_ARG);
  ZS_REQUIRE(num_experts >= 1 && num_experts <= 1024, ZS_ERR_SHAPE);
  ZS_REQUIRE(top_k >= 1 && top_k <= 32 && top_k <= num_experts, ZS_ERR_SHAPE);
  ZS_REQUIRE(num_tokens >= 0, ZS_ERR_SHAPE);
  ZS_BIND(gate_probs);
  if (num_tokens == 0) return ZS_OK;
  switch (probs_dtype) {
    case ZS_F32:
      return launch_gate_topk<float>(gate_probs, expert_biases, num_tokens, num_experts, top_k, topk_idx,
                                     topk_weight, stream);
    case ZS_BF16:
      return launch_gate_topk<__nv_bfloat16>(gate_probs, expert_biases, num_tokens, num_experts, top_k, topk_idx,
                                             topk_weight, stream);
    case ZS_F16:
      return launch_gate_topk<__half>(gate_probs, expert_biases, num_tokens, num_experts, top_k, topk_idx,
                                      topk_weight, stream);
  }
  return ZS_ERR_DTYPE;
}

extern "C" size_t zs_flatten_sort_count_workspace(int64_t n, int num_experts) {
  const int64_t nblk = (n + FSC_CHUNK - 1) / FSC_CHUNK;
  return (size_t)((nblk > 0 ? nblk : 1) * (num_experts + 1) * sizeof(int));
}

extern "C" int zs_flatten_sort_count(const int64_t* expert_idxs, int64_t n, int num_experts, int64_t* sorted_expert_idxs,
                                     int64_t* sorted_scattered_idxs, int64_t* expert_offsets, void* workspace,
                                     size_t workspace_bytes, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ZS_REQUIRE(expert_offsets, ZS_ERR_ARG);
  ZS_REQUIRE(n == 0 || (expert_idxs && sorted_expert_idxs && sorted_scattered_idxs), ZS_ERR_ARG);
  ZS_REQUIRE(num_experts >= 1 && num_experts <= 4096, ZS_ERR_SHAPE);
  ZS_REQUIRE(n >= 0 && n < ((int64_t)1 << 31), ZS_ERR_SHAPE);
  ZS_BIND(expert_offsets);
  if (n == 0) {
    ZS_CUDA_TRY(cudaMemsetAsync(expert_offsets, 0, sizeof(int64_t) * num_experts, stream));
    return ZS_OK;
  }
  ZS_REQUIRE(workspace != nullptr && workspace_bytes >= zs_flatten_sort_count_workspace(n, num_experts),
             ZS_ERR_WORKSPACE);
  const int nblk = (int)((n + FSC_CHUNK - 1) / FSC_CHUNK);
  const int B = num_experts + 1;
  int* hist = reinterpret_cast<int*>(workspace);
  fsc_hist_kernel<<<nblk, FSC_THREADS, B * sizeof(int), stream>>>(expert_idxs, n, num_experts, hist);
  ZS_CUDA_TRY(cudaGetLastError());
  const size_t scan_sh = (size_t)B * sizeof(int) * (1 + nblk);
  const int staged = scan_sh <= 96 * 1024;
  if (staged && scan_sh > 48 * 1024) {
    ZS_CUDA_TRY(cudaFuncSetAttribute(fsc_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)scan_sh));
  }
  fsc_scan_kernel<<<1, 1024, staged ? scan_sh : B * sizeof(int), stream>>>(hist, nblk, num_experts, expert_offsets,
                                                                           staged);
  ZS_CUDA_TRY(cudaGetLastError());
  const size_t sh = (size_t)B * sizeof(int) * (1 + FSC_THREADS / 32);
  if (sh > 48 * 1024) {
    ZS_CUDA_TRY(cudaFuncSetAttribute(fsc_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sh));
  }
  fsc_scatter_kernel<<<nblk, FSC_THREADS, sh, stream>>>(expert_idxs, n, num_experts, hist, sorted_expert_idxs,
                                                        sorted_scattered_idxs);
  ZS_CUDA_TRY(cudaGetLastError());
  return ZS_OK;
}

static int launch_count(const int64_t* x, const uint8_t* valid, int64_t n, int per_row, int minlength, int64_t* out,
                        cudaStream_t stream) {
  if (n == 0) return ZS_OK;
  int64_t blocks = (n + 1023) / 1024;
  if (blocks > 296) blocks = 296;
  const size_t sh = (size_t)minlength * sizeof(int);
  if (sh > 48 * 1024) {
    ZS_CUDA_TRY(cudaFuncSetAttribute(count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sh));
  }
  count_kernel<<<(unsigned)blocks, 1024, sh, stream>>>(x, valid, n, per_row, minlength, out);
  return cudaGetLastError() == cudaSuccess ? ZS_OK : ZS_ERR_CUDA;
}

extern "C" int zs_bincount(const int64_t* x, int64_t n, int minlength, int64_t* out, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ZS_REQUIRE(out && (n == 0 || x), ZS_ERR_ARG);
  ZS_REQUIRE(minlength >= 1 && minlength <= 49152 && n >= 0, ZS_ERR_SHAPE);
  ZS_BIND(out);
  ZS_CUDA_TRY(cudaMemsetAsync(out, 0, sizeof(int64_t) * minlength, stream));
  return launch_count(x, nullptr, n, 1, minlength, out, stream);
}

extern "C" int zs_expert_counts(const int64_t* topk_idx, const uint8_t* valid, int64_t num_tokens, int top_k,
                                int num_experts, int64_t* counts, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ZS_REQUIRE(counts && (num_tokens == 0 || topk_idx), ZS_ERR_ARG);
  ZS_REQUIRE(num_experts >= 1 && num_experts <= 49152 && top_k >= 1 && num_tokens >= 0, ZS_ERR_SHAPE);
  ZS_BIND(counts);
  return launch_count(topk_idx, valid, num_tokens * top_k, top_k, num_experts, counts, stream);
}

extern "C" int zs_bias_sign_update(const int64_t* counts, int num_experts, float update_rate, float* expert_biases,
                                   void* stream_) {
  ZS_REQUIRE(counts && expert_biases, ZS_ERR_ARG);
  ZS_REQUIRE(num_experts >= 1, ZS_ERR_SHAPE);
  ZS_BIND(counts);
  bias_sign_update_kernel<<<1, 256, 0, static_cast<cudaStream_t>(stream_)>>>(counts, num_experts, update_rate,
                                                                             expert_biases);
  return cudaGetLastError() == cudaSuccess ? ZS_OK : ZS_ERR_CUDA;
}

namespace zs {
// Gradient of topk_weight = L1-normalise(gate_probs[topk_idx]) with respect to
// gate_probs (the differentiable half of modeling/moe_gate.py:33-34):
//   s = sum_j |p_j|, D = max(s, eps)
//   dp_j = g_j / D - [s > eps] * sign(p_j) * (sum_i g_i p_i) / D^2
// scattered into a zero row of grad_probs [T, E].  One warp per token, f32.
template <typename T, typename G>
__global__ void gate_topk_backward_kernel(const T* __restrict__ probs, const int64_t* __restrict__ idx,
                                          const G* __restrict__ grad_w, T* __restrict__ grad_probs, int64_t num_tokens,
                                          int E, int k) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < num_tokens; t += warps) {
    int e = -1;
    float p = 0.f, g = 0.f;
    if (lane < k) {
      e = (int)idx[t * k + lane];
      if (e < 0 || e >= E) {
        record_error(ZS_DEVERR_INDEX);
        e = -1;
      } else {
        p = to_f32<T>(probs[t * E + e]);
        g = to_f32<G>(grad_w[t * k + lane]);
      }
    }
    float s = fabsf(p), dot = g * p;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      s += __shfl_xor_sync(0xffffffffu, s, off);
      dot += __shfl_xor_sync(0xffffffffu, dot, off);
    }
    const float eps = 1e-12f;
    const float D = fmaxf(s, eps);
    const float sg = p > 0.f ? 1.f : (p < 0.f ? -1.f : 0.f);
    const float dp = g / D - (s > eps ? sg * dot / (D * D) : 0.f);
    for (int c = lane; c < E; c += 32) {
      float v = 0.f;
      for (int j = 0; j < k; ++j) {
        const int ej = __shfl_sync(0xffffffffu, e, j);
        const float dj = __shfl_sync(0xffffffffu, dp, j);
        if (ej == c) v += dj;
      }
      grad_probs[t * E + c] = from_f32<T>(v);
    }
  }
}
}  // namespace zs

extern "C" int zs_moe_gate_topk_backward(const void* gate_probs, int probs_dtype, const int64_t* topk_idx,
                                         const void* grad_weight, int grad_dtype, int64_t num_tokens, int num_experts,
                                         int top_k, void* grad_probs, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ZS_REQUIRE(gate_probs && topk_idx && grad_weight && grad_probs, ZS_ERR_ARG);
  ZS_REQUIRE(num_experts >= 1 && num_experts <= 1024 && top_k >= 1 && top_k <= 32 && num_tokens >= 0, ZS_ERR_SHAPE);
  ZS_REQUIRE(grad_dtype == probs_dtype, ZS_ERR_DTYPE);
  ZS_BIND(gate_probs);
  if (num_tokens == 0) return ZS_OK;
  int64_t blocks = (num_tokens + 7) / 8;
  if (blocks > 148 * 32) blocks = 148 * 32;
#define ZS_GB(T)                                                                                                   \
  gate_topk_backward_kernel<T, T><<<(unsigned)blocks, 256, 0, stream>>>(                                           \
      reinterpret_cast<const T*>(gate_probs), topk_idx, reinterpret_cast<const T*>(grad_weight),                   \
      reinterpret_cast<T*>(grad_probs), num_tokens, num_experts, top_k)
  if (probs_dtype == ZS_F32)
    ZS_GB(float);
  else if (probs_dtype == ZS_BF16)
    ZS_GB(__nv_bfloat16);
  else if (probs_dtype == ZS_F16)
    ZS_GB(__half);
  else
    return ZS_ERR_DTYPE;
#undef ZS_GB
  return cudaGetLastError() == cudaSuccess ? ZS_OK : ZS_ERR_CUDA;
}

// ----------------------------------------------- allocation-free variant --
//
// Some callers cannot allocate device memory at the point where they route
// tokens: runtimes that own a fixed memory pool and forbid cudaMalloc after
// start-up, or plain C callers without an allocator.  For
// them zs_flatten_sort_count_noalloc keeps its scratch (the per-chunk expert
// histograms) in the fixed device array below instead of a caller workspace.
//
// The array is 1 MiB (ZS_FSC_NOALLOC_MAX_INTS ints) and exists on every GPU
// that loads this library until the process exits.  Host code cannot use the
// array's name as a device address (it names a host-side shadow), so the
// device address is looked up once per device with cudaGetSymbolAddress, with
// that device current, on the first call made on that device.
constexpr int64_t ZS_FSC_NOALLOC_MAX_INTS = (int64_t)1 << 18;
static __device__ __align__(256) int zs_fsc_noalloc_scratch[ZS_FSC_NOALLOC_MAX_INTS];

static int fsc_noalloc_scratch_ptr(void** out) {
  constexpr int MAX_DEVICES = 64;
  static std::mutex mu;
  static void* ptrs[MAX_DEVICES] = {};
  int dev = 0;
  ZS_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= MAX_DEVICES) return ZS_ERR_CUDA;
  std::lock_guard<std::mutex> lock(mu);
  if (ptrs[dev] == nullptr) {
    void* p = nullptr;
    ZS_CUDA_TRY(cudaGetSymbolAddress(&p, zs_fsc_noalloc_scratch));
    ptrs[dev] = p;
  }
  *out = ptrs[dev];
  return ZS_OK;
}

extern "C" int64_t zs_flatten_sort_count_noalloc_max_scratch_ints(void) { return ZS_FSC_NOALLOC_MAX_INTS; }

extern "C" int zs_flatten_sort_count_noalloc(const int64_t* expert_idxs, int64_t n, int num_experts,
                                             int64_t* sorted_expert_idxs, int64_t* sorted_scattered_idxs,
                                             int64_t* expert_offsets, void* stream) {
  ZS_REQUIRE(num_experts >= 1 && num_experts <= 4096 && n >= 0 && n < ((int64_t)1 << 31), ZS_ERR_SHAPE);
  ZS_BIND(expert_offsets);
  const size_t need = zs_flatten_sort_count_workspace(n, num_experts);
  if ((int64_t)(need / sizeof(int)) > ZS_FSC_NOALLOC_MAX_INTS) return ZS_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  const int rc = fsc_noalloc_scratch_ptr(&scratch);
  if (rc != ZS_OK) return rc;
  // Every histogram slot the sort reads is written by its first kernel in the
  // same call, so leftovers from an earlier call need no clearing.
  return zs_flatten_sort_count(expert_idxs, n, num_experts, sorted_expert_idxs, sorted_scattered_idxs, expert_offsets,
                               scratch, (size_t)ZS_FSC_NOALLOC_MAX_INTS * sizeof(int), stream);
}
