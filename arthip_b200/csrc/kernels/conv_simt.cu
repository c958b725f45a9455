// CUDA-core 3x3 convolution for the layers too narrow for the tensor-core tiling:
// the C==1 head conv (reference: direct_conv, src/common/hip_kernels.h:402-483), tails
// with a handful of output channels (fused DepthToSpace DCR + Clip + boundary layout and
// dtype: the reference's dts_kernel_2d / dts_kernel_in_f32 / cast_f16_to_f32_transpose,
// hip_kernels.h:553-670), and any other channel count.
//
// One thread computes one output pixel for a group of MG output channels; consecutive
// threads take consecutive channel groups of a pixel, so NHWC stores are contiguous.
// Weights live in shared memory as fp32 [tap][c][m]; accumulation is fp32.

#include <cstring>
#include <vector>

#include "kernels.h"

namespace ah {

namespace {

constexpr int kSimtThreads = 256;
constexpr int kSimtSmemWeights = 48 * 1024;

__device__ __forceinline__ float r16(float v) { return __half2float(__float2half_rn(v)); }

struct SimtArgs {
  const __half* in;
  const float* w;
  const float* bias;
  const __half* add1;
  const __half* add2;
  SimtOut out;
  int H, W, C, M, groups, act;
  int w_in_smem;
};

template <int MG, bool VEC8>
__global__ void __launch_bounds__(kSimtThreads) conv3x3_simt_kernel(const SimtArgs a) {
  extern __shared__ float sw[];
  const float* wsrc = a.w;
  if (a.w_in_smem) {
    const int n = 9 * a.C * a.M;
    for (int i = threadIdx.x; i < n; i += blockDim.x) sw[i] = a.w[i];
    __syncthreads();
    wsrc = sw;
  }
  // One grid row per image row; 32-bit index math (64-bit division is costly on GPUs).
  const int item = blockIdx.x * blockDim.x + threadIdx.x;
  if (item >= a.W * a.groups) return;
  const int g = item % a.groups;
  const int x = item / a.groups;
  const int y = blockIdx.y;
  const long long pix = static_cast<long long>(y) * a.W + x;
  const int mg0 = g * MG;
  const int nm = min(MG, a.M - mg0);

  float acc[MG];
#pragma unroll
  for (int j = 0; j < MG; ++j) acc[j] = 0.f;

  for (int ky = 0; ky < 3; ++ky) {
    const int yy = y + ky - 1;
    if (yy < 0 || yy >= a.H) continue;
    for (int kx = 0; kx < 3; ++kx) {
      const int xx = x + kx - 1;
      if (xx < 0 || xx >= a.W) continue;
      const int tap = ky * 3 + kx;
      const __half* src = a.in + (static_cast<long long>(yy) * a.W + xx) * a.C;
      const float* wt = wsrc + static_cast<long long>(tap) * a.C * a.M + mg0;
      if (VEC8) {
        for (int c8 = 0; c8 < a.C; c8 += 8) {
          const uint4 u = __ldg(reinterpret_cast<const uint4*>(src + c8));
          const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
          for (int j2 = 0; j2 < 4; ++j2) {
            const float2 xv = __half22float2(h[j2]);
            const float* w0 = wt + static_cast<long long>(c8 + 2 * j2) * a.M;
            const float* w1 = w0 + a.M;
#pragma unroll
            for (int j = 0; j < MG; ++j) {
              if (j < nm) {
                acc[j] = fmaf(xv.x, w0[j], acc[j]);
                acc[j] = fmaf(xv.y, w1[j], acc[j]);
              }
            }
          }
        }
      } else {
        for (int c = 0; c < a.C; ++c) {
          const float xv = __half2float(src[c]);
          const float* w0 = wt + static_cast<long long>(c) * a.M;
#pragma unroll
          for (int j = 0; j < MG; ++j)
            if (j < nm) acc[j] = fmaf(xv, w0[j], acc[j]);
        }
      }
    }
  }

  // Epilogue: bias, fp16 node rounding, activation, residual adds.
  const long long obase = pix * a.M + mg0;
#pragma unroll
  for (int j = 0; j < MG; ++j) {
    if (j >= nm) break;
    float t = r16(acc[j] + a.bias[mg0 + j]);
    if (a.act == kActRelu) {
      t = fmaxf(t, 0.f);
    } else if (a.act == kActSilu) {
      const float s = r16(sigmoid_fast(t));
      t = r16(t * s);
    }
    if (a.add1) t = r16(t + __half2float(a.add1[obase + j]));
    if (a.add2) t = r16(t + __half2float(a.add2[obase + j]));
    acc[j] = t;
  }

  const SimtOut& o = a.out;
  const int b = o.dts_b;
  if (b == 1 && !o.nchw && !o.fp32 && !o.clip) {
    __half* dst = static_cast<__half*>(o.ptr) + obase;
    if (nm == 8 && ((obase & 7) == 0)) {
      uint4 u;
      __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) h[j] = __floats2half2_rn(acc[2 * j], acc[2 * j + 1]);
      *reinterpret_cast<uint4*>(dst) = u;
    } else {
#pragma unroll
      for (int j = 0; j < MG; ++j)
        if (j < nm) dst[j] = __float2half_rn(acc[j]);
    }
    return;
  }
  // DepthToSpace (DCR: input channel m = (r*b + q)*Cout + c) and/or boundary layout.
  const int cout = a.M / (b * b);
  const long long Ho = static_cast<long long>(a.H) * b;
  const long long Wo = static_cast<long long>(a.W) * b;
#pragma unroll
  for (int j = 0; j < MG; ++j) {
    if (j >= nm) break;
    const int m = mg0 + j;
    const int rq = m / cout;
    const int c = m - rq * cout;
    const int r = rq / b;
    const int q = rq - r * b;
    const long long oy = static_cast<long long>(y) * b + r;
    const long long ox = static_cast<long long>(x) * b + q;
    float v = acc[j];
    if (o.clip) v = fminf(fmaxf(v, o.clip_lo), o.clip_hi);
    const long long idx = o.nchw ? ((static_cast<long long>(c) * Ho + oy) * Wo + ox) : ((oy * Wo + ox) * cout + c);
    if (o.fp32) static_cast<float*>(o.ptr)[idx] = v;
    else static_cast<__half*>(o.ptr)[idx] = __float2half_rn(v);
  }
}

// Single-input-channel head conv (C == 1, M % 8 == 0, plain NHWC fp16 output): each thread
// owns 8 output channels, keeps their 72 weights and 8 biases in registers, and walks
// kC1Run consecutive pixels of one row with a sliding 3x3 input window (3 new loads per
// pixel). Same accumulation order and epilogue as conv3x3_simt_kernel (tap-major fp32
// FMAs from zero, then + bias and the fp16 node rounding), so both give identical bits.
constexpr int kC1Run = 16;

__global__ void __launch_bounds__(kSimtThreads) conv3x3_c1_kernel(const SimtArgs a) {
  const int G = a.groups;  // M / 8
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  const int runs = (a.W + kC1Run - 1) / kC1Run;
  if (t >= runs * G) return;
  const int g = t % G;
  const int x0 = (t / G) * kC1Run;
  const int y = blockIdx.y;
  const int m0 = g * 8;
  float w[9][8], b[8];
#pragma unroll
  for (int tap = 0; tap < 9; ++tap)
#pragma unroll
    for (int j = 0; j < 8; ++j) w[tap][j] = __ldg(a.w + tap * a.M + m0 + j);
#pragma unroll
  for (int j = 0; j < 8; ++j) b[j] = __ldg(a.bias + m0 + j);
  const __half* row[3];
  bool rv[3];
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    const int yy = y + r - 1;
    rv[r] = yy >= 0 && yy < a.H;
    row[r] = a.in + static_cast<long long>(rv[r] ? yy : 0) * a.W;
  }
  auto ld = [&](int r, int xx) -> float {
    return (rv[r] && xx >= 0 && xx < a.W) ? __half2float(__ldg(row[r] + xx)) : 0.f;
  };
  float v[3][3];
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    v[r][0] = ld(r, x0 - 1);
    v[r][1] = ld(r, x0);
    v[r][2] = ld(r, x0 + 1);
  }
  const int xe = min(a.W, x0 + kC1Run);
  for (int x = x0; x < xe; ++x) {
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
    for (int r = 0; r < 3; ++r)
#pragma unroll
      for (int k = 0; k < 3; ++k)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = fmaf(v[r][k], w[r * 3 + k][j], acc[j]);
    const long long obase = (static_cast<long long>(y) * a.W + x) * a.M + m0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float t = r16(acc[j] + b[j]);
      if (a.act == kActRelu) t = fmaxf(t, 0.f);
      else if (a.act == kActSilu) t = r16(t * r16(sigmoid_fast(t)));
      acc[j] = t;
    }
    const __half* adds[2] = {a.add1, a.add2};
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      if (!adds[k]) continue;
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(adds[k] + obase));
      const __half* q = reinterpret_cast<const __half*>(&u);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = r16(acc[j] + __half2float(q[j]));
    }
    uint32_t h[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 o = __floats2half2_rn(acc[2 * i], acc[2 * i + 1]);
      h[i] = *reinterpret_cast<uint32_t*>(&o);
    }
    *reinterpret_cast<uint4*>(static_cast<__half*>(a.out.ptr) + obase) = make_uint4(h[0], h[1], h[2], h[3]);
#pragma unroll
    for (int r = 0; r < 3; ++r) {
      v[r][0] = v[r][1];
      v[r][1] = v[r][2];
      v[r][2] = ld(r, x + 2);
    }
  }
}

template <int MG, bool VEC8>
cudaError_t launch_simt(const SimtArgs& a, size_t smem, cudaStream_t s) {
  // Weights are staged only when they fit the default 48 KB dynamic shared memory, so no
  // function attribute (and nothing that is not stream-ordered) is needed here.
  const dim3 grid(static_cast<unsigned>((a.W * a.groups + kSimtThreads - 1) / kSimtThreads),
                  static_cast<unsigned>(a.H));
  conv3x3_simt_kernel<MG, VEC8><<<grid, kSimtThreads, smem, s>>>(a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t simt_conv_upload(const uint16_t* w_oihw, const float* bias, int C, int M, SimtConvWeights* out) {
  out->C = C;
  out->M = M;
  std::vector<float> w(static_cast<size_t>(9) * C * M);
  for (int m = 0; m < M; ++m)
    for (int c = 0; c < C; ++c)
      for (int t = 0; t < 9; ++t) {
        __half_raw hr;
        hr.x = w_oihw[(static_cast<size_t>(m) * C + c) * 9 + t];
        w[(static_cast<size_t>(t) * C + c) * M + m] = __half2float(__half(hr));
      }
  std::vector<float> b(M, 0.f);
  if (bias) std::memcpy(b.data(), bias, sizeof(float) * M);
  cudaError_t e = cudaMalloc(&out->w, w.size() * sizeof(float));
  if (e != cudaSuccess) return e;
  e = cudaMemcpy(out->w, w.data(), w.size() * sizeof(float), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return e;
  e = cudaMalloc(&out->bias, sizeof(float) * M);
  if (e != cudaSuccess) return e;
  e = cudaMemcpy(out->bias, b.data(), sizeof(float) * M, cudaMemcpyHostToDevice);
  if (e != cudaSuccess || !head_mma_supported(C, M)) return e;
  const std::vector<uint32_t> f = head_mma_fragments(w_oihw, bias, C, M);
  e = cudaMalloc(&out->bfrag, f.size() * sizeof(uint32_t));
  if (e != cudaSuccess) return e;
  return cudaMemcpy(out->bfrag, f.data(), f.size() * sizeof(uint32_t), cudaMemcpyHostToDevice);
}

void simt_conv_free(SimtConvWeights* w) {
  if (w->w) cudaFree(w->w);
  if (w->bias) cudaFree(w->bias);
  if (w->bfrag) cudaFree(w->bfrag);
  w->w = nullptr;
  w->bias = nullptr;
  w->bfrag = nullptr;
}

cudaError_t simt_conv_launch(const SimtConvWeights& w, const __half* in, int H, int W, const __half* add1,
                             const __half* add2, int act, const SimtOut& out, cudaStream_t s) {
  SimtArgs a;
  a.in = in;
  a.w = w.w;
  a.bias = w.bias;
  a.add1 = add1;
  a.add2 = add2;
  a.out = out;
  a.H = H;
  a.W = W;
  a.C = w.C;
  a.M = w.M;
  a.act = act;
  const size_t wbytes = static_cast<size_t>(9) * w.C * w.M * sizeof(float);
  a.w_in_smem = wbytes <= static_cast<size_t>(kSimtSmemWeights) ? 1 : 0;
  const size_t smem = a.w_in_smem ? wbytes : 0;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const bool plain = out.dts_b == 1 && !out.nchw && !out.fp32 && !out.clip;
  if (w.bfrag && plain && !add1 && !add2 && a16(out.ptr))
    return head_mma_launch(w.bfrag, w.bias, w.C, w.M, in, H, W, act, static_cast<__half*>(out.ptr), s);
  if (w.C == 1 && w.M % 8 == 0 && out.dts_b == 1 && !out.nchw && !out.fp32 && !out.clip && a16(out.ptr) &&
      a16(add1) && a16(add2)) {
    a.groups = w.M / 8;
    const int runs = (W + kC1Run - 1) / kC1Run;
    const dim3 grid(static_cast<unsigned>((runs * a.groups + kSimtThreads - 1) / kSimtThreads),
                    static_cast<unsigned>(H));
    conv3x3_c1_kernel<<<grid, kSimtThreads, 0, s>>>(a);
    return cudaGetLastError();
  }
  const bool vec8 = (w.C % 8 == 0) && a16(in);
  if (w.M <= 4) {
    a.groups = 1;
    return vec8 ? launch_simt<4, true>(a, smem, s) : launch_simt<4, false>(a, smem, s);
  }
  a.groups = (w.M + 7) / 8;
  return vec8 ? launch_simt<8, true>(a, smem, s) : launch_simt<8, false>(a, smem, s);
}

}  // namespace ah
