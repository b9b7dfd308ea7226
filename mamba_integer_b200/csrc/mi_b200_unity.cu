// mi_b200_unity.cu -- the library is compiled as this single translation unit
// so the per-device error word in mi_common.cuh has exactly one definition.
#include "mi_common.cuh"
#include "capi.cu"
#include "scan_i32.cu"
#include "rowops.cu"
#include "ssm.cu"
#include "gemm_i8.cu"
#include "decode.cu"
#include "train.cu"
#include "noalloc.cu"
