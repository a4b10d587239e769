// lib.cu -- single translation unit of libremora_b200.so.  The kernels share
// one device error word (rb::g_device_error), so they are compiled together.
#include "runtime.cuh"
#include "elementwise.cu"
#include "gemm.cu"
#include "gemm_f32.cu"
#include "attention.cu"
#include "moe.cu"
#include "moe_gemm.cu"
#include "moe_host.cu"
#include "moe_noalloc.cu"
#include "moe_ep_experts.cu"
#include "moe_ep.cu"
#include "dispatch.cu"
