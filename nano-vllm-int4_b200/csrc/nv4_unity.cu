// Single translation unit of libnv4 (see build_native.py).
#include "nv4_capi.cu"
#include "rht_quant.cu"
#include "w4a4_gemm.cu"
#include "w4a4_gemm_tc.cu"
#include "w4a16_gemm_tc.cu"
#include "w4a16_gemm.cu"
#include "peer_allreduce.cu"
#include "attention.cu"
