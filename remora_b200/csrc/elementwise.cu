// elementwise.cu -- the attention-epilogue elementwise chains and the seeded
// input generator.  HBM-bound: 128-bit coalesced loads/stores, grid-stride,
// grid sized to a multiple of the SM count, one HBM round trip per element.
#include "runtime.cuh"

namespace rb {

// maximumf semantics: NaN propagates, -0 and +0 both give +0.
__device__ __forceinline__ float relu_maximumf(float v) {
  return (v != v) ? v : (v > 0.0f ? v : 0.0f);
}

// x [rows, d], bias [d]; d % 4 == 0 and 16-byte aligned pointers.
__global__ void __launch_bounds__(256) k_relu_bias_v4(const float4* __restrict__ x,
                                                      const float4* __restrict__ bias,
                                                      float4* __restrict__ out, int64_t n4,
                                                      int64_t d4) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 v = __ldcs(x + i);
    float4 b = __ldg(bias + (i % d4));
    float4 r;
    r.x = relu_maximumf(__fadd_rn(v.x, b.x));
    r.y = relu_maximumf(__fadd_rn(v.y, b.y));
    r.z = relu_maximumf(__fadd_rn(v.z, b.z));
    r.w = relu_maximumf(__fadd_rn(v.w, b.w));
    __stcs(out + i, r);
  }
}

__global__ void __launch_bounds__(256) k_relu_bias_scalar(const float* __restrict__ x,
                                                          const float* __restrict__ bias,
                                                          float* __restrict__ out, int64_t n,
                                                          int64_t d) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = relu_maximumf(__fadd_rn(x[i], bias[i % d]));
}

__device__ __forceinline__ float scale_add_exp1(float s, float b, float scale) {
  return expf(__fadd_rn(__fmul_rn(s, scale), b));
}

// Two float4 per thread per iteration so that each SM keeps enough bytes in
// flight to cover HBM latency.
__global__ void __launch_bounds__(256) k_scale_add_exp_v4(const float4* __restrict__ s,
                                                          const float4* __restrict__ b,
                                                          float4* __restrict__ out, int64_t n4,
                                                          float scale) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + stride < n4; i += 2 * stride) {
    float4 s0 = __ldcs(s + i), b0 = __ldcs(b + i);
    float4 s1 = __ldcs(s + i + stride), b1 = __ldcs(b + i + stride);
    float4 r0, r1;
    r0.x = scale_add_exp1(s0.x, b0.x, scale);
    r0.y = scale_add_exp1(s0.y, b0.y, scale);
    r0.z = scale_add_exp1(s0.z, b0.z, scale);
    r0.w = scale_add_exp1(s0.w, b0.w, scale);
    r1.x = scale_add_exp1(s1.x, b1.x, scale);
    r1.y = scale_add_exp1(s1.y, b1.y, scale);
    r1.z = scale_add_exp1(s1.z, b1.z, scale);
    r1.w = scale_add_exp1(s1.w, b1.w, scale);
    __stcs(out + i, r0);
    __stcs(out + i + stride, r1);
  }
  if (i < n4) {
    float4 s0 = __ldcs(s + i), b0 = __ldcs(b + i), r0;
    r0.x = scale_add_exp1(s0.x, b0.x, scale);
    r0.y = scale_add_exp1(s0.y, b0.y, scale);
    r0.z = scale_add_exp1(s0.z, b0.z, scale);
    r0.w = scale_add_exp1(s0.w, b0.w, scale);
    __stcs(out + i, r0);
  }
}

__global__ void k_scale_add_exp_scalar(const float* __restrict__ s, const float* __restrict__ b,
                                       float* __restrict__ out, int64_t lo, int64_t n,
                                       float scale) {
  int64_t i = lo + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = scale_add_exp1(s[i], b[i], scale);
}

inline int ew_grid(int64_t work_items, int threads) {
  int64_t want = (work_items + threads - 1) / threads;
  int64_t cap = (int64_t)num_sms() * 8;  // 8 CTAs of 256 threads per SM
  int64_t g = want < cap ? want : cap;
  return (int)(g > 0 ? g : 1);
}

// ------------------------------------------------------------ generator
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__device__ __forceinline__ double unit01(uint64_t key, uint64_t ctr) {
  uint64_t b = mix64(key + (ctr + 1) * 0x9E3779B97F4A7C15ull);
  return ((double)(b >> 11) + 0.5) * (1.0 / 9007199254740992.0);
}

__device__ __forceinline__ uint16_t f32_to_bf16_rne(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

__global__ void k_fill(void* out, int64_t n, int dtype, int normal, uint64_t key, double p0,
                       double p1) {
  const double two_pi = 6.283185307179586476925286766559;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    double v;
    if (normal) {
      double u1 = unit01(key, 2 * (uint64_t)i), u2 = unit01(key, 2 * (uint64_t)i + 1);
      v = p0 + p1 * (sqrt(-2.0 * log(u1)) * cos(two_pi * u2));
    } else {
      v = p0 + (p1 - p0) * unit01(key, (uint64_t)i);
    }
    float f = (float)v;
    if (dtype == 0)
      static_cast<float*>(out)[i] = f;
    else
      static_cast<uint16_t*>(out)[i] = f32_to_bf16_rne(f);
  }
}

}  // namespace rb

using namespace rb;

extern "C" int remora_b200_relu_bias_f32(const float* x, const float* bias, float* out,
                                         int64_t rows, int64_t d, void* stream) {
  clear_error();
  RB_CHECK_ARG(rows >= 0 && d > 0, "relu_bias: rows=%lld d=%lld", (long long)rows, (long long)d);
  int64_t n = rows * d;
  if (n == 0) return REMORA_B200_OK;
  RB_CHECK_ARG(x && bias && out, "relu_bias: null pointer");
  cudaStream_t st = as_stream(stream);
  if (d % 4 == 0 && aligned16(x) && aligned16(bias) && aligned16(out)) {
    int64_t n4 = n / 4;
    k_relu_bias_v4<<<ew_grid(n4, 256), 256, 0, st>>>(reinterpret_cast<const float4*>(x),
                                                    reinterpret_cast<const float4*>(bias),
                                                    reinterpret_cast<float4*>(out), n4, d / 4);
  } else {
    k_relu_bias_scalar<<<ew_grid(n, 256), 256, 0, st>>>(x, bias, out, n, d);
  }
  RB_LAUNCH_CHECK();
  return REMORA_B200_OK;
}

extern "C" int remora_b200_scale_add_exp_f32(const float* s, const float* b, float* out,
                                             int64_t n, float scale, void* stream) {
  clear_error();
  RB_CHECK_ARG(n >= 0, "scale_add_exp: n=%lld", (long long)n);
  if (n == 0) return REMORA_B200_OK;
  RB_CHECK_ARG(s && b && out, "scale_add_exp: null pointer");
  cudaStream_t st = as_stream(stream);
  int64_t head = 0;
  if (aligned16(s) && aligned16(b) && aligned16(out)) {
    int64_t n4 = n / 4;
    if (n4 > 0)
      k_scale_add_exp_v4<<<ew_grid((n4 + 1) / 2, 256), 256, 0, st>>>(
          reinterpret_cast<const float4*>(s), reinterpret_cast<const float4*>(b),
          reinterpret_cast<float4*>(out), n4, scale);
    head = n4 * 4;
  }
  if (head < n) {
    int64_t rest = n - head;
    k_scale_add_exp_scalar<<<(unsigned)((rest + 255) / 256), 256, 0, st>>>(s, b, out, head, n,
                                                                         scale);
  }
  RB_LAUNCH_CHECK();
  return REMORA_B200_OK;
}

static int fill_impl(void* out, int64_t n, int dtype, int normal, uint64_t key, double p0,
                     double p1, void* stream) {
  clear_error();
  RB_CHECK_ARG(out && n >= 0 && (dtype == 0 || dtype == 1), "fill: bad arguments");
  if (n == 0) return REMORA_B200_OK;
  k_fill<<<ew_grid(n, 256), 256, 0, as_stream(stream)>>>(out, n, dtype, normal, key, p0, p1);
  RB_LAUNCH_CHECK();
  return REMORA_B200_OK;
}

extern "C" int remora_b200_fill_normal(void* out, int64_t n, int dtype, uint64_t key,
                                       double mean, double sigma, void* stream) {
  return fill_impl(out, n, dtype, 1, key, mean, sigma, stream);
}

extern "C" int remora_b200_fill_uniform(void* out, int64_t n, int dtype, uint64_t key,
                                        double lo, double hi, void* stream) {
  return fill_impl(out, n, dtype, 0, key, lo, hi, stream);
}
