// All-reduce of data-parallel gradients over NVLink peer memory, moved by the
// copy engines instead of SM kernels.
//
// The grouped GEMMs of the backward pass hold one persistent CTA on every SM,
// so a collective whose kernels need SMs (NCCL's) slows the GEMM it runs beside.
// Here every byte crosses NVLink in cudaMemcpyAsync peer copies (copy engines,
// no SMs); the only SM work is one short reduction kernel per step and
// single-thread flag kernels.
//
// World N, a buffer of `count` elements split into N chunks of c elements
// (c a multiple of 8).  Every rank holds, mapped into every peer through CUDA
// IPC, a receive buffer of N slots of c elements, a reduced-chunk buffer of c
// elements and an int32 flag table [3][N]:
//   flags[0][s] = last step whose chunk from rank s landed in my receive slot s
//   flags[1][s] = last step whose reduced chunk rank s has published
//   flags[2][s] = last step rank s has finished reducing (its slot for me is free)
// One step s (>= 1) on `stream`, rank r:
//   1. wait flags[2][*] >= s - 1            (my previous sends were consumed)
//   2. copy chunk p of my data to rank p's receive slot r, for every p != r
//   3. set flags[0][r] = s on every peer
//   4. wait flags[0][*] >= s
//   5. reduce: chunk r = scale * sum over ranks in rank order (f32), written to
//      my data and my reduced-chunk buffer
//   6. set flags[2][r] = s and flags[1][r] = s on every peer
//   7. wait flags[1][*] >= s
//   8. copy every peer's reduced chunk into my data
// Only rank r computes chunk r and the sum runs in rank order, so every rank
// ends with bit-identical data.  Waits are bounded (about a second of clock64);
// on expiry they record ZS_DEVERR_TIMEOUT_PEER and return.
#include "zs_common.cuh"

namespace zs {
namespace comm {

constexpr int MAX_RANKS = 16;

struct FlagPtrs {
  int* p[MAX_RANKS];
};

// Bounded wait until flags[i] >= target for every i in [0, n) other than skip.
__global__ void ce_wait_kernel(const int* flags, int n, int skip, int target) {
  const int i = threadIdx.x;
  if (i >= n || i == skip) return;
  const long long t0 = clock64();
  unsigned ns = 64;
  while (true) {
    int v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(flags + i) : "memory");
    if (v >= target) return;
    if (clock64() - t0 > (long long)ZS_WAIT_TIMEOUT_CYCLES) {
      record_error(ZS_DEVERR_TIMEOUT_PEER);
      return;
    }
    __nanosleep(ns);
    if (ns < 2048) ns <<= 1;
  }
}

// Every earlier operation of the stream (the peer copies) is complete when this
// runs; publish `value` into flag slot `slot` of every peer but `skip`.
__global__ void ce_signal_kernel(FlagPtrs flags, int n, int skip, int slot, int value, int slot2) {
  const int i = threadIdx.x;
  if (i >= n || i == skip) return;
  __threadfence_system();
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(flags.p[i] + slot), "r"(value) : "memory");
  if (slot2 >= 0)
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(flags.p[i] + slot2), "r"(value) : "memory");
}

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

// out[j] = scale * sum_{s < n} (s == me ? mine[j] : recv[s * slot + j]), s ascending,
// written to out0 and out1; j in [0, len).  8 elements per thread-iteration.
template <typename T>
__global__ void ce_reduce_kernel(T* out0, T* __restrict__ out1, const T* mine, const T* __restrict__ recv,
                                 int64_t slot, int n, int me, int64_t len, float scale) {
  const int64_t groups = (len + 7) / 8;
  for (int64_t gi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; gi < groups;
       gi += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j0 = gi * 8;
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    const bool full = j0 + 8 <= len;
    for (int s = 0; s < n; ++s) {
      const T* src = (s == me ? mine : recv + s * slot) + j0;
      if (full && sizeof(T) == 2) {
        const uint4 u = *reinterpret_cast<const uint4*>(src);
        const T* v = reinterpret_cast<const T*>(&u);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += to_f<T>(v[e]);
      } else if (full) {
        const float4 a = *reinterpret_cast<const float4*>(src);
        const float4 b = *reinterpret_cast<const float4*>(src + 4);
        acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
        acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (j0 + e < len) acc[e] += to_f<T>(src[e]);
      }
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      if (j0 + e < len) {
        const T v = from_f32<T>(acc[e] * scale);
        out0[j0 + e] = v;
        out1[j0 + e] = v;
      }
    }
  }
}

}  // namespace comm
}  // namespace zs

using namespace zs;

extern "C" int zs_ipc_handle_size(void) { return (int)sizeof(cudaIpcMemHandle_t); }

// CUDA IPC handle of the allocation holding `ptr`, and ptr's byte offset in it.
extern "C" int zs_ipc_export(const void* ptr, void* handle_out, int64_t* offset_out) {
  ZS_REQUIRE(ptr && handle_out && offset_out, ZS_ERR_ARG);
  ZS_BIND(ptr);
  static PFN_cuMemGetAddressRange_v3020 range_fn = nullptr;
  if (range_fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return ZS_ERR_CUDA;
    range_fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range_fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return ZS_ERR_CUDA;
  cudaIpcMemHandle_t h;
  ZS_CUDA_TRY(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = (int64_t)(reinterpret_cast<uintptr_t>(ptr) - (uintptr_t)base);
  return ZS_OK;
}

// Map a peer's allocation (from zs_ipc_export) into this process on `device`;
// *ptr_out = mapped base + offset, *base_out = the mapping to pass to zs_ipc_close.
extern "C" int zs_ipc_open(const void* handle, int64_t offset, int device, void** ptr_out, void** base_out) {
  ZS_REQUIRE(handle && ptr_out && base_out && offset >= 0, ZS_ERR_ARG);
  ZS_CUDA_TRY(cudaSetDevice(device));
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  ZS_CUDA_TRY(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
  *base_out = base;
  *ptr_out = static_cast<char*>(base) + offset;
  return ZS_OK;
}

extern "C" int zs_ipc_close(void* base) {
  ZS_REQUIRE(base, ZS_ERR_ARG);
  ZS_CUDA_TRY(cudaIpcCloseMemHandle(base));
  return ZS_OK;
}

extern "C" int64_t zs_ce_allreduce_chunk(int64_t count, int world) {
  if (count < 1 || world < 1) return 0;
  const int64_t c = (count + world - 1) / world;
  return (c + 7) / 8 * 8;
}

extern "C" int zs_ce_allreduce(void* data, int64_t count, int dtype, int rank, int world, void* const* recv,
                               void* const* red, int* const* flags, int step, float scale, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ZS_REQUIRE(data && recv && red && flags, ZS_ERR_ARG);
  ZS_REQUIRE(dtype == ZS_BF16 || dtype == ZS_F32, ZS_ERR_DTYPE);
  ZS_REQUIRE(world >= 1 && world <= comm::MAX_RANKS && rank >= 0 && rank < world && count >= 1 && step >= 1,
             ZS_ERR_SHAPE);
  for (int p = 0; p < world; ++p) ZS_REQUIRE(recv[p] && red[p] && flags[p], ZS_ERR_ARG);
  ZS_REQUIRE(reinterpret_cast<uintptr_t>(data) % 16 == 0, ZS_ERR_ALIGN);
  ZS_BIND(data);
  const size_t es = dtype == ZS_BF16 ? 2 : 4;
  const int64_t c = zs_ce_allreduce_chunk(count, world);
  auto chunk_len = [&](int p) -> int64_t {
    const int64_t lo = (int64_t)p * c;
    return lo >= count ? 0 : (count - lo < c ? count - lo : c);
  };
  char* d = static_cast<char*>(data);
  int* my_flags = flags[rank];
  comm::FlagPtrs fp{};
  for (int p = 0; p < world; ++p) fp.p[p] = flags[p];
  // 1. my sends of the previous step were consumed
  if (world > 1) {
    comm::ce_wait_kernel<<<1, 32, 0, stream>>>(my_flags + 2 * world, world, rank, step - 1);
    ZS_CUDA_TRY(cudaGetLastError());
  }
  // 2. chunk p -> rank p's receive slot `rank`
  for (int p = 0; p < world; ++p) {
    if (p == rank || chunk_len(p) == 0) continue;
    ZS_CUDA_TRY(cudaMemcpyAsync(static_cast<char*>(recv[p]) + (size_t)rank * c * es, d + (size_t)p * c * es,
                                (size_t)chunk_len(p) * es, cudaMemcpyDeviceToDevice, stream));
  }
  if (world > 1) {
    // 3. data landed; 4. wait for every peer's chunk
    comm::ce_signal_kernel<<<1, 32, 0, stream>>>(fp, world, rank, 0 * world + rank, step, -1);
    ZS_CUDA_TRY(cudaGetLastError());
    comm::ce_wait_kernel<<<1, 32, 0, stream>>>(my_flags + 0 * world, world, rank, step);
    ZS_CUDA_TRY(cudaGetLastError());
  }
  // 5. reduce my chunk in rank order
  const int64_t len = chunk_len(rank);
  if (len > 0) {
    int64_t blocks = (len / 8 + 255) / 256;
    if (blocks > 148 * 4) blocks = 148 * 4;
    if (blocks < 1) blocks = 1;
    if (dtype == ZS_BF16) {
      auto* o = reinterpret_cast<__nv_bfloat16*>(d) + (size_t)rank * c;
      comm::ce_reduce_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, stream>>>(
          o, static_cast<__nv_bfloat16*>(red[rank]), o, static_cast<const __nv_bfloat16*>(recv[rank]), c, world,
          rank, len, scale);
    } else {
      auto* o = reinterpret_cast<float*>(d) + (size_t)rank * c;
      comm::ce_reduce_kernel<float><<<(unsigned)blocks, 256, 0, stream>>>(
          o, static_cast<float*>(red[rank]), o, static_cast<const float*>(recv[rank]), c, world, rank, len, scale);
    }
    ZS_CUDA_TRY(cudaGetLastError());
  }
  if (world > 1) {
    // 6. my receive slots are free and my reduced chunk is published; 7. wait for the peers'
    comm::ce_signal_kernel<<<1, 32, 0, stream>>>(fp, world, rank, 2 * world + rank, step, 1 * world + rank);
    ZS_CUDA_TRY(cudaGetLastError());
    comm::ce_wait_kernel<<<1, 32, 0, stream>>>(my_flags + 1 * world, world, rank, step);
    ZS_CUDA_TRY(cudaGetLastError());
  }
  // 8. pull every peer's reduced chunk
  for (int p = 0; p < world; ++p) {
    if (p == rank || chunk_len(p) == 0) continue;
    ZS_CUDA_TRY(cudaMemcpyAsync(d + (size_t)p * c * es, red[p], (size_t)chunk_len(p) * es, cudaMemcpyDeviceToDevice,
                                stream));
  }
  return ZS_OK;
}
