// Library-level entry points: version, error strings and the device error word.
#include "zs_common.cuh"

extern "C" int zs_version(void) { return 1; }

extern "C" const char* zs_error_string(int code) {
  switch (code) {
    case ZS_OK: return "ok";
    case ZS_ERR_ARG: return "null pointer or invalid argument";
    case ZS_ERR_SHAPE: return "sizes inconsistent or outside the supported range";
    case ZS_ERR_DTYPE: return "unsupported dtype";
    case ZS_ERR_ALIGN: return "pointer or row pitch not 16-byte aligned (TMA requirement)";
    case ZS_ERR_CUDA: return "CUDA runtime or driver call failed";
    case ZS_ERR_WORKSPACE: return "workspace missing or too small";
    case ZS_ERR_LAYOUT: return "stride pattern not supported";
    case ZS_ERR_SCRATCH_LIMIT: return "problem larger than the fixed scratch of the allocation-free entry point";
  }
  return "unknown zs error";
}

extern "C" int zs_device_error_get(int* out, void* stream) {
  ZS_REQUIRE(out, ZS_ERR_ARG);
  ZS_CUDA_TRY(cudaMemcpyFromSymbolAsync(out, zs_device_error, sizeof(int), 0, cudaMemcpyDeviceToHost,
                                        static_cast<cudaStream_t>(stream)));
  ZS_CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  return ZS_OK;
}

extern "C" int zs_device_error_clear(void* stream) {
  static const int zero = 0;
  ZS_CUDA_TRY(cudaMemcpyToSymbolAsync(zs_device_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice,
                                      static_cast<cudaStream_t>(stream)));
  ZS_CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  return ZS_OK;
}

extern "C" int zs_last_cuda_error(void) { return zs_last_cuda_error_ref(); }
