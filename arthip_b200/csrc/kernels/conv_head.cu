// Tensor-core head conv for inputs with very few channels (C <= 4: the luma head C = 1,
// the chroma / RGB heads C = 3), the reference's direct_conv (src/common/hip_kernels.h:
// 402-483). The whole 3x3xC receptive field of a pixel is one K <= 64 operand row, so per
// 16-pixel tile the conv is KS = ceil(9C/16) mma.sync m16n8k16 steps per 8 output
// channels (fp16 operands, fp32 accumulation). A CUDA-core formulation spends ~70 FMA
// instructions per pixel and output-channel octet and is issue-bound; here the tensor
// cores do the products and the warps only stage operands and store results.
//
// Block = a 256-pixel segment of 4 output rows (4 warps x 4 tiles of 16 per row). The six
// input rows it reads (+1 pixel halo each side, zero outside the frame) are staged in
// shared memory; each lane gathers its A-fragment elements from there. Weight fragments
// are packed on the host in the mma.sync B layout and held in registers. Results go
// through a padded per-warp staging tile so every global store is a coalesced 16 bytes.
// Epilogue as the other conv kernels: + bias, fp16 rounding of the conv node, ReLU / SiLU.

#include <cstring>
#include <vector>

#include "kernels.h"

namespace ah {

namespace {

constexpr int kHeadThreads = 128;
constexpr int kHeadSeg = 256;              // output pixels per block
constexpr int kHeadRow = kHeadSeg + 2;     // staged input pixels per row
constexpr int kHeadMaxC = 4;
constexpr int kHeadRows = 4;               // output rows per block

struct HeadArgs {
  const __half* in;
  const uint32_t* bfrag;
  const float* bias;
  __half* out;
  int H, W, C, M, act;
};

__device__ __forceinline__ float r16(float v) { return __half2float(__float2half_rn(v)); }

__device__ __forceinline__ uint32_t pack_h2(__half lo, __half hi) {
  return static_cast<uint32_t>(__half_as_ushort(lo)) | (static_cast<uint32_t>(__half_as_ushort(hi)) << 16);
}

__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int C, int NT>
__global__ void __launch_bounds__(kHeadThreads) conv3x3_head_mma_kernel(const HeadArgs a) {
  constexpr int KS = (9 * C + 15) / 16;
  constexpr int kIn = kHeadRows + 2;  // staged input rows
  __shared__ __half s_in[kIn * kHeadRow * C];
  __shared__ __align__(16) uint32_t s_stage[kHeadThreads / 32][16 * (NT * 4 + 4)];
  const int y0 = blockIdx.y * kHeadRows;
  const int xb = blockIdx.x * kHeadSeg;
  // Stage rows y0-1 .. y0+kHeadRows, pixels xb-1 .. xb+256 (zero outside the frame: the
  // conv padding).
  for (int i = threadIdx.x; i < kIn * kHeadRow * C; i += kHeadThreads) {
    const int r = i / (kHeadRow * C);
    const int rem = i - r * (kHeadRow * C);
    const int gx = xb - 1 + rem / C;
    const int gy = y0 - 1 + r;
    __half v = __float2half(0.f);
    if (gy >= 0 && gy < a.H && gx >= 0 && gx < a.W)
      v = a.in[(static_cast<long long>(gy) * a.W + gx) * C + rem % C];
    s_in[i] = v;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  // This lane's K indices: 16s + 2t + {0, 1, 8, 9}; k = tap * C + c, tap = ky * 3 + kx.
  int koff[KS][4];
#pragma unroll
  for (int s = 0; s < KS; ++s)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int k = 16 * s + 2 * t + (e & 1) + (e >> 1) * 8;
      const int tap = k / C, c = k - tap * C;
      koff[s][e] = k < 9 * C ? ((tap / 3) * kHeadRow + tap % 3) * C + c : -1;
    }
  uint32_t b[NT][KS][2];
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int s = 0; s < KS; ++s) {
      const uint2 v = __ldg(reinterpret_cast<const uint2*>(a.bfrag) + (j * KS + s) * 32 + lane);
      b[j][s][0] = v.x;
      b[j][s][1] = v.y;
    }
  float2 bias[NT];
#pragma unroll
  for (int j = 0; j < NT; ++j) bias[j] = __ldg(reinterpret_cast<const float2*>(a.bias + 8 * j + 2 * t));
  __syncthreads();

  constexpr int kStride = NT * 4 + 4;  // staging row: M/2 words + 4 (bank spread)
  uint32_t* stage = s_stage[warp];
  const __half2 zero2 = __float2half2_rn(0.f);
  for (int rr = 0; rr < kHeadRows; ++rr) {
    const int y = y0 + rr;
    if (y >= a.H) break;
    for (int tile = 0; tile < 4; ++tile) {
      const int xl = warp * 64 + tile * 16;  // tile's first pixel, relative to xb
      if (xb + xl >= a.W) break;
      float acc[NT][4];
#pragma unroll
      for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
#pragma unroll
      for (int s = 0; s < KS; ++s) {
        __half v[2][4];
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
          for (int e = 0; e < 4; ++e)
            v[r][e] = koff[s][e] >= 0 ? s_in[rr * kHeadRow * C + koff[s][e] + (xl + g + 8 * r) * C]
                                      : __float2half(0.f);
        const uint32_t af[4] = {pack_h2(v[0][0], v[0][1]), pack_h2(v[1][0], v[1][1]),
                                pack_h2(v[0][2], v[0][3]), pack_h2(v[1][2], v[1][3])};
#pragma unroll
        for (int j = 0; j < NT; ++j) mma_16816(acc[j], af, b[j][s][0], b[j][s][1]);
      }
      // Epilogue: lane holds pixels g and g+8, channels 8j + 2t, +1. The fp16 store
      // rounding is the conv node's rounding; ReLU commutes with it.
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          __half2 h;
          if (a.act == kActSilu) {
            float o[2];
#pragma unroll
            for (int i = 0; i < 2; ++i) {
              const float v = r16(acc[j][2 * r + i] + (i ? bias[j].y : bias[j].x));
              o[i] = r16(v * r16(sigmoid_fast(v)));
            }
            h = __floats2half2_rn(o[0], o[1]);
          } else {
            h = __floats2half2_rn(acc[j][2 * r] + bias[j].x, acc[j][2 * r + 1] + bias[j].y);
            if (a.act == kActRelu) h = __hmax2(h, zero2);
          }
          stage[(g + 8 * r) * kStride + 4 * j + t] = *reinterpret_cast<uint32_t*>(&h);
        }
      __syncwarp();
      // 16 pixels x NT 16-byte chunks, consecutive lanes on consecutive chunks.
#pragma unroll
      for (int i = 0; i < (16 * NT) / 32; ++i) {
        const int ch = lane + 32 * i;
        const int p = ch / NT, jj = ch - p * NT;
        const int px = xb + xl + p;
        if (px < a.W) {
          const uint4 v = *reinterpret_cast<const uint4*>(stage + p * kStride + 4 * jj);
          *reinterpret_cast<uint4*>(a.out + (static_cast<long long>(y) * a.W + px) * a.M + 8 * jj) = v;
        }
      }
      __syncwarp();
    }
  }
}

template <int C>
cudaError_t launch_c(const HeadArgs& a, int NT, cudaStream_t s) {
  const dim3 grid(static_cast<unsigned>((a.W + kHeadSeg - 1) / kHeadSeg),
                  static_cast<unsigned>((a.H + kHeadRows - 1) / kHeadRows));
  switch (NT) {
    case 4: conv3x3_head_mma_kernel<C, 4><<<grid, kHeadThreads, 0, s>>>(a); break;
    case 8: conv3x3_head_mma_kernel<C, 8><<<grid, kHeadThreads, 0, s>>>(a); break;
    case 12: conv3x3_head_mma_kernel<C, 12><<<grid, kHeadThreads, 0, s>>>(a); break;
    default: conv3x3_head_mma_kernel<C, 16><<<grid, kHeadThreads, 0, s>>>(a); break;
  }
  return cudaGetLastError();
}

}  // namespace

bool head_mma_supported(int C, int M) { return C >= 1 && C <= kHeadMaxC && M % 32 == 0 && M >= 32 && M <= 128; }

std::vector<uint32_t> head_mma_fragments(const uint16_t* w_oihw, int C, int M) {
  const int KS = (9 * C + 15) / 16, NT = M / 8;
  std::vector<uint32_t> f(static_cast<size_t>(NT) * KS * 32 * 2, 0u);
  auto bk = [&](int k, int n) -> uint32_t {  // B[k][n] = w[n][c][tap], k = tap * C + c
    if (k >= 9 * C) return 0u;
    const int tap = k / C, c = k % C;
    return w_oihw[(static_cast<size_t>(n) * C + c) * 9 + tap];
  };
  for (int j = 0; j < NT; ++j)
    for (int s = 0; s < KS; ++s)
      for (int l = 0; l < 32; ++l) {
        const int n = 8 * j + l / 4, k0 = 16 * s + 2 * (l % 4);
        uint32_t* d = &f[((static_cast<size_t>(j) * KS + s) * 32 + l) * 2];
        d[0] = bk(k0, n) | (bk(k0 + 1, n) << 16);
        d[1] = bk(k0 + 8, n) | (bk(k0 + 9, n) << 16);
      }
  return f;
}

cudaError_t head_mma_launch(const uint32_t* bfrag, const float* bias, int C, int M, const __half* in, int H, int W,
                            int act, __half* out, cudaStream_t s) {
  HeadArgs a;
  a.in = in;
  a.bfrag = bfrag;
  a.bias = bias;
  a.out = out;
  a.H = H;
  a.W = W;
  a.C = C;
  a.M = M;
  a.act = act;
  const int NT = M / 8;
  switch (C) {
    case 1: return launch_c<1>(a, NT, s);
    case 2: return launch_c<2>(a, NT, s);
    case 3: return launch_c<3>(a, NT, s);
    default: return launch_c<4>(a, NT, s);
  }
}

}  // namespace ah
