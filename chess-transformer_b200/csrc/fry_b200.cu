// The whole library as one translation unit: the device status word (common.cuh) has a single definition, and no
// relocatable device code or device link step is needed. Built by chess-transformer_b200/build.py into libfry_b200.so.
#include "gemm.cu"
#include "rows.cu"
#include "attention.cu"
#include "attention64.cu"
#include "heads.cu"
#include "gptq.cu"
#include "health.cu"
#include "abi.cu"
#include "noalloc.cu"
#include "lanes.cu"
