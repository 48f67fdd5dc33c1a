// fence_cuda.cu — the single CUDA translation unit of libfence_b200.so. Device globals (the
// device error word) and every kernel live in one module, so no relocatable device code is needed.
#include "gemv.cu"
#include "rgemv.cu"
#include "step.cu"
#include "ops.cu"
#include "attention_static.cu"
#include "sampler_dev.cu"
#include "prefill.cu"
#include "engine.cu"
