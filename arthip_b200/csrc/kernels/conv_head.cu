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
//
// The luma head (C = 1) has a kernel of its own, shaped by what bounded the general one
// (about 15 warp instructions per output pixel: operand gathers of single fp16 values, a
// per-element epilogue and a per-lane store path, at five resident blocks per SM):
//  * the staged input is held as vertical pairs (row j, row j + 1) in one 32-bit word,
//    and the K order of the 3x3 taps is chosen so that each A-fragment register is one
//    such pair: (ky 0, ky 1) at kx = 0..2, then (ky 2, zero weight) at kx = 0..2. Every
//    operand load is then one aligned 32-bit shared load;
//  * K slot 12 holds a constant 1 and the matching B row the bias (fp16, as the conv's
//    weights), so the MMA adds the bias exactly and the epilogue has no bias adds;
//  * fp16 rounding and ReLU in one cvt.rn.relu.f16x2.f32 per channel pair, stmatrix into a
//    128B-swizzled staging tile (conflict-free), and one TMA store per 16-pixel tile,
//    double-buffered per warp.
// One warp per output row of a block of eight (four for M > 64) and 128 pixels.

#include <cstring>
#include <string>
#include <vector>

#include "fp16_host.h"
#include "kernels.h"
#include "ptx.cuh"

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

// ---------------------------------------------------------------------------
// C = 1 head
// ---------------------------------------------------------------------------
constexpr int kH1Px = 128;      // output pixels per block row
constexpr int kH1Pitch = 136;   // words per staged pair row: 2 * 136 % 32 == 16, so the two
                                // pair rows one fragment load reads fall in disjoint banks
constexpr int kH1Staged = kH1Px + 2;

struct Head1Args {
  CUtensorMap map64;  // output [H][W][M], box {64, 16, 1}, 128B swizzle (64-channel chunks)
  CUtensorMap map32;  // box {32, 16, 1}, 64B swizzle (a trailing 32-channel chunk)
  const __half* in;
  const uint32_t* bfrag;
  int H, W;
};

__device__ __forceinline__ void stmatrix_x4(uint32_t addr, const uint32_t (&r)[4]) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3])
               : "memory");
}

// fp16 rounding of a channel pair (the conv node's output) and the activation; low half =
// first channel.
template <int ACT>
__device__ __forceinline__ uint32_t head1_pack(float lo, float hi) {
  uint32_t d;
  if constexpr (ACT == kActRelu) {
    asm("cvt.rn.relu.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  } else if constexpr (ACT == kActSilu) {
    const float v0 = r16(lo), v1 = r16(hi);
    const __half2 h = __floats2half2_rn(r16(v0 * r16(sigmoid_fast(v0))), r16(v1 * r16(sigmoid_fast(v1))));
    d = *reinterpret_cast<const uint32_t*>(&h);
  } else {
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  }
  return d;
}

// Byte offset of (pixel row p, 8-channel slab) in a 16-pixel staging tile laid out as the
// TMA store boxes read it: 64-channel chunks of 16 x 128 B (128B swizzle), then a 32-channel
// chunk of 16 x 64 B (64B swizzle).
template <int M>
__device__ __forceinline__ uint32_t head1_stage_off(int p, int slab) {
  constexpr int N64 = M / 64;
  const int ci = slab >> 3;
  if (ci < N64) return ci * 2048 + p * 128 + (((slab & 7) ^ (p & 7)) << 4);
  const int c = slab - 8 * N64;
  return N64 * 2048 + p * 64 + ((c ^ ((p >> 1) & 3)) << 4);
}

template <int NT, int ACT>
__global__ void __launch_bounds__(32 * (NT <= 8 ? 8 : 4), NT <= 8 ? 5 : 6)
    conv3x3_head1_kernel(const __grid_constant__ Head1Args a) {
  constexpr int M = 8 * NT;
  constexpr int ROWS = NT <= 8 ? 8 : 4;  // output rows per block = warps
  constexpr int PAIRS = ROWS + 2;        // staged pair rows (row j, row j + 1)
  constexpr int N64 = M / 64, N32 = (M % 64) / 32;
  constexpr int TILE = 16 * M * 2;       // one 16-pixel staging tile
  __shared__ uint32_t s_vp[PAIRS * kH1Pitch];
  __shared__ __align__(1024) uint8_t s_stage[ROWS][2][TILE];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int x0 = blockIdx.x * kH1Px, y0 = blockIdx.y * ROWS;

  uint32_t b[NT][2];
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const uint2 v = __ldg(reinterpret_cast<const uint2*>(a.bfrag) + j * 32 + lane);
    b[j][0] = v.x;
    b[j][1] = v.y;
  }
  // Pair row j holds input rows y0 - 1 + j (low half) and y0 + j (high half), pixels
  // x0 - 1 .. x0 + 128; zero outside the frame (the conv padding). The high half of the last
  // pair row is only ever multiplied by a zero weight: it is staged as 0. Two threads per
  // staged column, each loading the input rows of half of the pair rows (all its loads
  // issued before the first use).
  constexpr int HP = PAIRS / 2;  // pair rows per half
  const unsigned short* in = reinterpret_cast<const unsigned short*>(a.in);
  for (int u = threadIdx.x; u < 2 * kH1Staged; u += 32 * ROWS) {
    const int half = u >= kH1Staged ? 1 : 0;
    const int px = u - half * kH1Staged;
    const int gx = x0 - 1 + px;
    const bool colok = gx >= 0 && gx < a.W;
    const int j0 = half * HP;
    uint32_t v[HP + 1];
#pragma unroll
    for (int r = 0; r <= HP; ++r) {
      const int gy = y0 - 1 + j0 + r;
      v[r] = (colok && j0 + r < PAIRS && gy >= 0 && gy < a.H) ? in[static_cast<long long>(gy) * a.W + gx] : 0u;
    }
#pragma unroll
    for (int r = 0; r < HP; ++r) s_vp[(j0 + r) * kH1Pitch + px] = v[r] | (v[r + 1] << 16);
  }
  __syncthreads();
  const int y = y0 + warp;
  if (y >= a.H) return;
  // A fragment: a0/a1 = K pair t of pixels g / g + 8, a2/a3 = K pair t + 4. Pairs 0..2:
  // (ky 0, ky 1) at kx = pair; pairs 3..5: (ky 2, 0) at kx = pair - 3; pair 6: the constant
  // 1 (bias); pair 7: zero.
  const int offA = (t < 3 ? warp * kH1Pitch + t : (warp + 2) * kH1Pitch) + g;
  const int offB = (warp + 2) * kH1Pitch + t + 1 + g;
  const uint32_t constB = t == 2 ? 0x3C00u : 0u;
  // stmatrix.x4 row address of this lane: matrix lane / 8 = (slab j + lane / 16, pixels
  // 0-7 or 8-15), row lane % 8
  const int p = ((lane >> 3) & 1) * 8 + (lane & 7);
  const int hi = lane >> 4;
  const uint32_t stage0 = ptx::smem_u32(&s_stage[warp][0][0]);
  int issued = 0;
  for (int xt = 0; xt < kH1Px; xt += 16) {
    const int px0 = x0 + xt;
    if (px0 >= a.W) break;
    uint32_t af[4];
    af[0] = s_vp[offA + xt];
    af[1] = s_vp[offA + xt + 8];
    if (t < 2) {
      af[2] = s_vp[offB + xt];
      af[3] = s_vp[offB + xt + 8];
    } else {
      af[2] = af[3] = constB;
    }
    const int sb = (xt >> 4) & 1;
    if (issued >= 2) {  // the store that read this buffer two tiles ago has finished reading it
      if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
      __syncwarp();
    }
    const uint32_t buf = stage0 + sb * TILE;
#pragma unroll
    for (int j = 0; j < NT; j += 2) {
      float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
      mma_16816(d0, af, b[j][0], b[j][1]);
      mma_16816(d1, af, b[j + 1][0], b[j + 1][1]);
      const uint32_t r[4] = {head1_pack<ACT>(d0[0], d0[1]), head1_pack<ACT>(d0[2], d0[3]),
                             head1_pack<ACT>(d1[0], d1[1]), head1_pack<ACT>(d1[2], d1[3])};
      stmatrix_x4(buf + head1_stage_off<M>(p, j + hi), r);
    }
    ptx::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
#pragma unroll
      for (int ci = 0; ci < N64; ++ci) ptx::tma_store_3d(&a.map64, buf + ci * 2048, ci * 64, px0, y);
      if constexpr (N32 > 0) ptx::tma_store_3d(&a.map32, buf + N64 * 2048, N64 * 64, px0, y);
      ptx::bulk_commit_group();
    }
    ++issued;
  }
  if (lane == 0) ptx::bulk_wait_group0();
  __syncwarp();
}

template <int NT>
cudaError_t launch_head1_nt(const Head1Args& h, int act, cudaStream_t s) {
  constexpr int ROWS = NT <= 8 ? 8 : 4;
  const dim3 grid(static_cast<unsigned>((h.W + kH1Px - 1) / kH1Px), static_cast<unsigned>((h.H + ROWS - 1) / ROWS));
  switch (act) {
    case kActRelu: conv3x3_head1_kernel<NT, kActRelu><<<grid, 32 * ROWS, 0, s>>>(h); break;
    case kActSilu: conv3x3_head1_kernel<NT, kActSilu><<<grid, 32 * ROWS, 0, s>>>(h); break;
    default: conv3x3_head1_kernel<NT, kActNone><<<grid, 32 * ROWS, 0, s>>>(h); break;
  }
  return cudaGetLastError();
}

cudaError_t launch_head1(const uint32_t* bfrag, int M, const __half* in, int H, int W, int act, __half* out,
                         cudaStream_t s) {
  Head1Args h;
  std::memset(&h, 0, sizeof(h));
  std::string err;
  if (M >= 64 && !encode_nhwc_map(&h.map64, out, M, W, H, 64, 16, &err)) return cudaErrorInvalidValue;
  if (M % 64 == 32 && !encode_nhwc_map(&h.map32, out, M, W, H, 32, 16, &err)) return cudaErrorInvalidValue;
  h.in = in;
  h.bfrag = bfrag;
  h.H = H;
  h.W = W;
  switch (M / 8) {
    case 4: return launch_head1_nt<4>(h, act, s);
    case 8: return launch_head1_nt<8>(h, act, s);
    case 12: return launch_head1_nt<12>(h, act, s);
    default: return launch_head1_nt<16>(h, act, s);
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

std::vector<uint32_t> head_mma_fragments(const uint16_t* w_oihw, const float* bias, int C, int M) {
  const int NT = M / 8;
  if (C == 1) {
    // K = 2 * pair + e: pairs 0..2 = (ky = e, kx = pair); pairs 3..5 = (ky 2, kx = pair - 3)
    // for e = 0 and zero for e = 1; pair 6, e = 0: the bias (A holds a constant 1 there).
    auto bk = [&](int k, int n) -> uint32_t {
      const int pr = k >> 1, e = k & 1;
      if (pr < 3) return w_oihw[static_cast<size_t>(n) * 9 + e * 3 + pr];
      if (pr < 6) return e == 0 ? w_oihw[static_cast<size_t>(n) * 9 + 6 + (pr - 3)] : 0u;
      if (pr == 6 && e == 0) return bias ? FloatToHalfRNE(bias[n]) : 0u;
      return 0u;
    };
    std::vector<uint32_t> f(static_cast<size_t>(NT) * 32 * 2, 0u);
    for (int j = 0; j < NT; ++j)
      for (int l = 0; l < 32; ++l) {
        const int n = 8 * j + l / 4, k0 = 2 * (l % 4);
        uint32_t* d = &f[(static_cast<size_t>(j) * 32 + l) * 2];
        d[0] = bk(k0, n) | (bk(k0 + 1, n) << 16);
        d[1] = bk(k0 + 8, n) | (bk(k0 + 9, n) << 16);
      }
    return f;
  }
  const int KS = (9 * C + 15) / 16;
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
    case 1: return launch_head1(bfrag, M, in, H, W, act, out, s);
    case 2: return launch_c<2>(a, NT, s);
    case 3: return launch_c<3>(a, NT, s);
    default: return launch_c<4>(a, NT, s);
  }
}

}  // namespace ah
