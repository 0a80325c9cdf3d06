// Single translation unit for libzs.so: the kernels share one device-global
// error word, so they are compiled together rather than with separate device
// linking.
#include "zs_gemm.cu"
#include "zs_moe.cu"
#include "zs_routing.cu"
#include "zs_norm.cu"
#include "zs_attn.cu"
#include "zs_muon.cu"
#include "zs_adam.cu"
#include "zs_comm.cu"
#include "zs_sparse.cu"
#include "zs_api.cu"
