// The whole library is one translation unit: device helpers and the device
// error flag in common.cuh are defined once and inlined everywhere without
// relocatable device code.
#include "host_util.cu"
#include "gemm.cu"
#include "attention_tc.cu"
#include "attention.cu"
#include "attention_noalloc.cu"
#include "elementwise.cu"
#include "capi.cu"
#include "engine.cu"
