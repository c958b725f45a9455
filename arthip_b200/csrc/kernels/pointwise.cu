// Pointwise fallbacks for graph nodes that cannot be fused into a conv epilogue, the
// standalone DepthToSpace, and the NCHW <-> NHWC boundary conversions.
// Reference counterparts: unary_kernel / binary_kernel / dts_kernel / transpose_f16 /
// cast_f32_to_f16_transpose / cast_f16_to_f32_transpose (src/common/hip_kernels.h:486-670).
// Every node result is rounded to fp16, as an fp16 ONNX tensor is.

#include "kernels.h"

namespace ah {

namespace {

constexpr int kThreads = 256;

unsigned blocks_for(size_t n) { return static_cast<unsigned>((n + kThreads - 1) / kThreads); }

__global__ void unary_kernel(const __half* __restrict__ in, __half* __restrict__ out, size_t n, int op, float lo,
                             float hi) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float x = __half2float(in[i]);
  float y;
  if (op == kSigmoid) y = sigmoid_fast(x);
  else if (op == kRelu) y = fmaxf(x, 0.f);
  else y = fminf(fmaxf(x, lo), hi);
  out[i] = __float2half_rn(y);
}

__global__ void binary_kernel(const __half* __restrict__ a, const __half* __restrict__ b, __half* __restrict__ out,
                              size_t n, int op) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float x = __half2float(a[i]);
  const float y = __half2float(b[i]);
  out[i] = __float2half_rn(op == kMul ? x * y : x + y);
}

// One thread per output element. DCR: output (c, h*b + r, w*b + q) <- input channel
// (r*b + q)*Cout + c.
__global__ void dts_kernel(const __half* __restrict__ in, int H, int W, int Cin, SimtOut o) {
  const int b = o.dts_b;
  const int cout = Cin / (b * b);
  const long long Ho = static_cast<long long>(H) * b, Wo = static_cast<long long>(W) * b;
  const long long n = Ho * Wo * cout;
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  long long oy, ox;
  int c;
  if (o.nchw) {
    c = static_cast<int>(i / (Ho * Wo));
    const long long rem = i - static_cast<long long>(c) * Ho * Wo;
    oy = rem / Wo;
    ox = rem - oy * Wo;
  } else {
    c = static_cast<int>(i % cout);
    const long long p = i / cout;
    oy = p / Wo;
    ox = p - oy * Wo;
  }
  const long long y = oy / b, x = ox / b;
  const int r = static_cast<int>(oy - y * b), q = static_cast<int>(ox - x * b);
  float v = __half2float(in[(y * W + x) * Cin + (r * b + q) * cout + c]);
  if (o.clip) v = fminf(fmaxf(v, o.clip_lo), o.clip_hi);
  if (o.fp32) static_cast<float*>(o.ptr)[i] = v;
  else static_cast<__half*>(o.ptr)[i] = __float2half_rn(v);
}

__global__ void nchw_to_nhwc_kernel(const void* __restrict__ in, int in_fp32, __half* __restrict__ out, int C,
                                    long long HW) {
  const long long p = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (p >= HW) return;
  for (int c = 0; c < C; ++c) {
    const long long s = static_cast<long long>(c) * HW + p;
    const __half v = in_fp32 ? __float2half_rn(static_cast<const float*>(in)[s]) : static_cast<const __half*>(in)[s];
    out[p * C + c] = v;
  }
}

__global__ void nhwc_to_nchw_kernel(const __half* __restrict__ in, void* __restrict__ out, int out_fp32, int C,
                                    long long HW) {
  const long long p = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (p >= HW) return;
  for (int c = 0; c < C; ++c) {
    const __half v = in[p * C + c];
    const long long d = static_cast<long long>(c) * HW + p;
    if (out_fp32) static_cast<float*>(out)[d] = __half2float(v);
    else static_cast<__half*>(out)[d] = v;
  }
}

}  // namespace

cudaError_t unary_launch(const __half* in, __half* out, size_t n, int op, float lo, float hi, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  unary_kernel<<<blocks_for(n), kThreads, 0, s>>>(in, out, n, op, lo, hi);
  return cudaGetLastError();
}

cudaError_t binary_launch(const __half* a, const __half* b, __half* out, size_t n, int op, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  binary_kernel<<<blocks_for(n), kThreads, 0, s>>>(a, b, out, n, op);
  return cudaGetLastError();
}

cudaError_t dts_launch(const __half* in, int H, int W, int Cin, const SimtOut& o, cudaStream_t s) {
  const size_t n = static_cast<size_t>(H) * W * Cin;
  if (n == 0) return cudaSuccess;
  dts_kernel<<<blocks_for(n), kThreads, 0, s>>>(in, H, W, Cin, o);
  return cudaGetLastError();
}

cudaError_t nchw_to_nhwc_launch(const void* in, int in_fp32, __half* out, int C, int H, int W, cudaStream_t s) {
  const long long HW = static_cast<long long>(H) * W;
  nchw_to_nhwc_kernel<<<blocks_for(static_cast<size_t>(HW)), kThreads, 0, s>>>(in, in_fp32, out, C, HW);
  return cudaGetLastError();
}

cudaError_t nhwc_to_nchw_launch(const __half* in, void* out, int out_fp32, int C, int H, int W, cudaStream_t s) {
  const long long HW = static_cast<long long>(H) * W;
  nhwc_to_nchw_kernel<<<blocks_for(static_cast<size_t>(HW)), kThreads, 0, s>>>(in, out, out_fp32, C, HW);
  return cudaGetLastError();
}

}  // namespace ah
