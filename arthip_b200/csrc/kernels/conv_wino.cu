// Winograd F(2x2,3x3) 3x3 convolution on the sm_100a tensor cores, for 64 -> 64 channel
// layers: the reference's winograd_conv (src/common/hip_kernels.h:143-396) and its weight
// transform (src/vapoursynth/hip_engine.cc:972-1009), redesigned for tcgen05 / TMEM / TMA.
//
// Numerics follow the reference: U = G g G^T in fp32 rounded to fp16 (host), the input
// transform V = B^T d B in fp16 arithmetic (column combinations first, then rows, each
// rounded), the 16 per-point channel contractions on the tensor cores with fp32
// accumulation, and the output transform A^T M A in fp32. The epilogue is the engine's:
// + bias, one fp16 rounding (the Conv node), ReLU / SiLU, residual adds rounded to fp16.
// fp16 V and U carry ~2^-11 relative error each, so this path is opt-in (engine conv
// algorithm "winograd"); the default direct implicit GEMM has exact fp16 products.
//
// Work unit: 128 Winograd tiles = 2 tile rows x 64 tile columns = 4 output rows x 128
// output pixels, which is one MMA M of 128 rows (TMEM lanes). Each CTA computes 32 of the
// 64 output channels (gridDim.y = 2), so all 16 points' accumulators, 16 x 32 fp32
// columns, fill exactly the 512 TMEM columns. Per unit:
//  * producer (warp 0): per 16-channel chunk kc, six TMA row loads (input rows y0-1 ..
//    y0+4, pixels x0-1 .. x0+128; the TMA unit zero-fills outside the frame: the padding)
//    into a double-buffered input slot;
//  * transform (warps 2-5, one tile per thread, warp w on TMEM lane quarter w - 2): per
//    chunk and half (points of rows p = 0,1, then p = 2,3), V for 8 points x 16 channels
//    with half2 arithmetic, stored as the MMA A operand (K-major, 32-byte rows, 32B
//    swizzle) into a double-buffered V slot;
//  * MMA (warp 1, one thread): per V slot, 8 MMAs 128 x 32 x 16 (A = V, B = U of the point
//    and chunk, resident in shared memory, 128B swizzle), accumulating point p into TMEM
//    columns 32p..32p+31;
//  * epilogue (warps 6-9, warp w on TMEM lane quarter w % 4): per 4-channel group, the 16 points' accumulators from TMEM, the
//    output transform, bias, rounding, activation, into a per-warp staging tile; then the
//    accumulators are released and the staging tile goes out with coalesced 16-byte
//    stores after the residual adds.
// Every wait is time-bounded; a timeout sets the status word instead of hanging.

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../fp16_host.h"
#include "kernels.h"
#include "ptx.cuh"

namespace ah {

namespace {

constexpr int kWThreads = 320;
constexpr int kWUnitRows = 4;      // output rows per unit
constexpr int kWUnitPx = 128;      // output pixels per unit row
constexpr int kWInRows = 6;        // input rows per unit
constexpr int kWBoxPx = 130;       // input pixels per row (unit + halo)
constexpr int kWRowPitch = 4224;   // bytes per staged input row (130 x 32 B, padded to 128 B)
constexpr int kWInSlot = 25600;    // one chunk's six rows (6 x 4224, 1024-aligned)
constexpr int kWVSlot = 32768;     // 8 points x 128 rows x 32 B
constexpr int kWUBytes = 65536;    // 16 points x 32 rows x 128 B
constexpr int kWStagePitch = 80;   // bytes per staged output pixel (32 channels + pad)
constexpr int kWStageWarp = 2 * 64 * kWStagePitch;  // 2 rows x 64 pixels
constexpr int kWOffU = 0;
constexpr int kWOffV = kWOffU + kWUBytes;
constexpr int kWOffIn = kWOffV + 2 * kWVSlot;
constexpr int kWOffStage = kWOffIn + 2 * kWInSlot;
constexpr int kWOffBars = kWOffStage + 4 * kWStageWarp;
constexpr int kWSmem = kWOffBars + 256 + 1024;  // barriers + alignment slack

struct WinoArgs {
  CUtensorMap in_map;  // fp16 NHWC input, box {16 channels, 130 pixels, 1 row}, no swizzle
  const uint8_t* upack;  // [2 halves][16 points][32 rows][128 B], 128B-swizzled K-major
  const float* bias;     // 64
  const __half* add1;
  const __half* add2;
  __half* out;
  uint32_t* status;
  int H, W, act;
  int units_x;
  long long units;
  unsigned long long wait_limit_ns;
};

// Byte offset of 16-byte granule j of row r in a 32B-swizzled K-major tile with 32-byte
// rows (granule index XOR bit 2 of the row), and in a 128B-swizzled one with 128-byte rows
// (granule index XOR row % 8): the layouts the MMA descriptors read, for tiles that start
// on a 1024-byte boundary.
__host__ __device__ constexpr uint32_t swz32(uint32_t r, uint32_t j) { return r * 32u + ((j ^ ((r >> 2) & 1u)) << 4); }
__host__ __device__ constexpr uint32_t swz128(uint32_t r, uint32_t j) { return r * 128u + ((j ^ (r & 7u)) << 4); }

__device__ __forceinline__ float r16f(float v) { return __half2float(__float2half_rn(v)); }

__device__ __forceinline__ uint32_t h2u(__half2 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ __half2 u2h(uint32_t v) { return *reinterpret_cast<__half2*>(&v); }

__device__ __forceinline__ void tmem_ld_x4(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr)
               : "memory");
}

// Column combinations of one staged input row (4 pixels, 8 channels as 4 half2 each):
// t = (c0 - c2, c1 + c2, c2 - c1, c1 - c3), every result rounded to fp16.
__device__ __forceinline__ void col_combos(const uint4 (&c)[4], uint32_t (&t)[4][4]) {
  const uint32_t* c0 = reinterpret_cast<const uint32_t*>(&c[0]);
  const uint32_t* c1 = reinterpret_cast<const uint32_t*>(&c[1]);
  const uint32_t* c2 = reinterpret_cast<const uint32_t*>(&c[2]);
  const uint32_t* c3 = reinterpret_cast<const uint32_t*>(&c[3]);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    t[0][k] = h2u(__hsub2(u2h(c0[k]), u2h(c2[k])));
    t[1][k] = h2u(__hadd2(u2h(c1[k]), u2h(c2[k])));
    t[2][k] = h2u(__hsub2(u2h(c2[k]), u2h(c1[k])));
    t[3][k] = h2u(__hsub2(u2h(c1[k]), u2h(c3[k])));
  }
}

__global__ void __launch_bounds__(kWThreads, 1) conv3x3_wino_kernel(const __grid_constant__ WinoArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sU = smem + kWOffU;
  uint8_t* sV = smem + kWOffV;
  uint8_t* sIn = smem + kWOffIn;
  uint8_t* sStage = smem + kWOffStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kWOffBars);
  uint64_t* in_full = bars;       // [2]
  uint64_t* in_empty = bars + 2;  // [2]
  uint64_t* v_full = bars + 4;    // [2]
  uint64_t* v_empty = bars + 6;   // [2]
  uint64_t* d_full = bars + 8;
  uint64_t* d_empty = bars + 9;
  uint64_t* wbar = bars + 10;
  uint64_t* donebar = bars + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int half = blockIdx.y;  // output channels 32 * half .. + 31
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(ptx::smem_u32(&in_full[i]), 1);
      ptx::mbar_init(ptx::smem_u32(&in_empty[i]), 4);
      ptx::mbar_init(ptx::smem_u32(&v_full[i]), 4);
      ptx::mbar_init(ptx::smem_u32(&v_empty[i]), 1);
    }
    ptx::mbar_init(ptx::smem_u32(d_full), 1);
    ptx::mbar_init(ptx::smem_u32(d_empty), 4);
    ptx::mbar_init(ptx::smem_u32(wbar), 1);
    ptx::mbar_init(ptx::smem_u32(donebar), 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) ptx::prefetch_tensormap(&a.in_map);
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_u32(tmem_slot), 512);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const unsigned long long lim = a.wait_limit_ns;

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      ptx::mbar_arrive_expect_tx(ptx::smem_u32(wbar), kWUBytes);
      for (int part = 0; part < 4; ++part)  // four 16 KB bulk copies of this half's U
        ptx::bulk_load(ptx::smem_u32(sU + part * 16384),
                       a.upack + static_cast<size_t>(half) * kWUBytes + part * 16384, 16384, ptx::smem_u32(wbar));
      ptx::griddep_wait();  // the input comes from the previous layer
      uint32_t cnt = 0;
      bool ok = true;
      for (long long u = blockIdx.x; u < a.units && ok; u += gridDim.x) {
        const int ux = static_cast<int>(u % a.units_x), uy = static_cast<int>(u / a.units_x);
        const int x0 = ux * kWUnitPx - 1, y0 = uy * kWUnitRows - 1;
        for (int kc = 0; kc < 4; ++kc, ++cnt) {
          const uint32_t s = cnt & 1u, ph = (cnt >> 1) & 1u;
          if (!ptx::mbar_wait(ptx::smem_u32(&in_empty[s]), ph ^ 1u, abort_flag, lim)) {
            ok = false;
            break;
          }
          const uint32_t fb = ptx::smem_u32(&in_full[s]);
          ptx::mbar_arrive_expect_tx(fb, kWInRows * kWBoxPx * 32);
          const uint32_t dst = ptx::smem_u32(sIn + s * kWInSlot);
          for (int r = 0; r < kWInRows; ++r) ptx::tma_load_3d(dst + r * kWRowPitch, &a.in_map, fb, kc * 16, x0, y0 + r);
        }
      }
      // No TMA write in flight at exit: wait (bounded) for the last loads.
      volatile int never_abort = 0;
      const uint32_t first = cnt > 2u ? cnt - 2u : 0u;
      for (uint32_t j = first; j < cnt; ++j)
        ptx::mbar_wait(ptx::smem_u32(&in_full[j & 1u]), (j >> 1) & 1u, &never_abort, lim);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      bool ok = ptx::mbar_wait(ptx::smem_u32(wbar), 0, abort_flag, lim);
      const uint32_t idesc = ptx::idesc_f16_f32(128, 32);
      const uint32_t v_lo0 = ptx::desc_lo(ptx::smem_u32(sV));
      const uint32_t u_lo0 = ptx::desc_lo(ptx::smem_u32(sU));
      const uint32_t a_hi = ptx::desc_hi(256, 6);   // 32B swizzle, 8 rows x 32 B
      const uint32_t b_hi = ptx::desc_hi(1024, 2);  // 128B swizzle, 8 rows x 128 B
      uint32_t vcnt = 0, ucnt = 0;
      for (long long u = blockIdx.x; u < a.units && ok; u += gridDim.x, ++ucnt) {
        ok = ptx::mbar_wait(ptx::smem_u32(d_empty), (ucnt & 1u) ^ 1u, abort_flag, lim);
        if (!ok) break;
        ptx::tc_fence_after();
        for (int kc = 0; kc < 4 && ok; ++kc)
          for (int h = 0; h < 2 && ok; ++h, ++vcnt) {
            const uint32_t s = vcnt & 1u;
            ok = ptx::mbar_wait(ptx::smem_u32(&v_full[s]), (vcnt >> 1) & 1u, abort_flag, lim);
            if (!ok) break;
            ptx::tc_fence_after();
#pragma unroll
            for (int pl = 0; pl < 8; ++pl) {
              const int p = 8 * h + pl;
              const uint32_t d = tmem_base + static_cast<uint32_t>(p * 32);
              const uint32_t alo = v_lo0 + ((s * kWVSlot + pl * 4096) >> 4);
              const uint32_t blo = u_lo0 + ((p * 4096 + kc * 32) >> 4);
              if (kc == 0) {
                const uint64_t ad = (static_cast<uint64_t>(a_hi) << 32) | alo;
                const uint64_t bd = (static_cast<uint64_t>(b_hi) << 32) | blo;
                ptx::mma_f16_ss(d, ad, bd, idesc, 0);
              } else {
                ptx::mma_f16_ss_acc(d, alo, a_hi, blo, b_hi, idesc);
              }
            }
            ptx::mma_commit(ptx::smem_u32(&v_empty[s]));
          }
        if (ok) ptx::mma_commit(ptx::smem_u32(d_full));
      }
      ptx::mma_commit(ptx::smem_u32(donebar));
      volatile int never_abort = 0;
      ptx::mbar_wait(ptx::smem_u32(donebar), 0, &never_abort, lim);
    }
    __syncwarp();
  } else if (warp < 6) {
    // ---------------- input transform ----------------
    const int q = warp - 2;
    const int t = 32 * q + lane;       // tile = TMEM lane = A row
    const int tr = t >> 6, tc = t & 63;
    uint32_t icnt = 0, vcnt = 0;
    bool ok = true;
    for (long long u = blockIdx.x; u < a.units && ok; u += gridDim.x) {
      for (int kc = 0; kc < 4 && ok; ++kc, ++icnt) {
        const uint32_t is = icnt & 1u;
        int w_ok = 1;
        if (lane == 0)
          w_ok = ptx::mbar_wait(ptx::smem_u32(&in_full[is]), (icnt >> 1) & 1u, abort_flag, lim) ? 1 : 0;
        w_ok = __shfl_sync(0xffffffffu, w_ok, 0);
        if (!w_ok) {
          ok = false;
          break;
        }
        const uint8_t* in = sIn + is * kWInSlot + (2 * tr) * kWRowPitch + (2 * tc) * 32;
        for (int h = 0; h < 2; ++h, ++vcnt) {
          const uint32_t vs = vcnt & 1u;
          if (lane == 0)
            w_ok = ptx::mbar_wait(ptx::smem_u32(&v_empty[vs]), ((vcnt >> 1) & 1u) ^ 1u, abort_flag, lim) ? 1 : 0;
          w_ok = __shfl_sync(0xffffffffu, w_ok, 0);
          if (!w_ok) {
            ok = false;
            break;
          }
          uint8_t* vdst = sV + vs * kWVSlot;
#pragma unroll
          for (int c8 = 0; c8 < 2; ++c8) {  // 8 channels at a time
            // Column combinations of the three input rows this half needs (rows 0-2 for
            // points p = 0, 1; rows 1-3 for p = 2, 3).
            uint32_t tt[3][4][4];
#pragma unroll
            for (int i = 0; i < 3; ++i) {
              const uint8_t* row = in + (h + i) * kWRowPitch + c8 * 16;
              uint4 c[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) c[j] = *reinterpret_cast<const uint4*>(row + j * 32);
              col_combos(c, tt[i]);
            }
            // Row combinations: h = 0: p0 = r0 - r2, p1 = r1 + r2; h = 1: p2 = r2 - r1,
            // p3 = r1 - r3 (rows relative to the half's first row: r_{h+i} = tt[i]).
#pragma unroll
            for (int pp = 0; pp < 2; ++pp)
#pragma unroll
              for (int qq = 0; qq < 4; ++qq) {
                uint32_t v[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                  __half2 x;
                  if (h == 0) x = pp == 0 ? __hsub2(u2h(tt[0][qq][k]), u2h(tt[2][qq][k]))
                                          : __hadd2(u2h(tt[1][qq][k]), u2h(tt[2][qq][k]));
                  else x = pp == 0 ? __hsub2(u2h(tt[1][qq][k]), u2h(tt[0][qq][k]))
                                   : __hsub2(u2h(tt[0][qq][k]), u2h(tt[2][qq][k]));
                  v[k] = h2u(x);
                }
                const int pl = pp * 4 + qq;  // point within the half
                *reinterpret_cast<uint4*>(vdst + pl * 4096 + swz32(t, c8)) = make_uint4(v[0], v[1], v[2], v[3]);
              }
          }
          ptx::fence_proxy_async_smem();  // the tensor core reads these generic writes
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(&v_full[vs]));
        }
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(&in_empty[is]));
      }
    }
  } else {
    // ---------------- epilogue ----------------
    ptx::griddep_wait();  // residual operands and the output buffer belong to earlier layers
    // A warp may read only TMEM lane quarter warp % 4: warps 6, 7, 8, 9 take the tiles
    // (lanes) 64-95, 96-127, 0-31, 32-63.
    const int q = warp & 3;
    const int tr = q >> 1;
    uint8_t* stage = sStage + q * kWStageWarp;
    const int n0 = 32 * half;
    uint32_t ucnt = 0;
    bool ok = true;
    for (long long u = blockIdx.x; u < a.units && ok; u += gridDim.x, ++ucnt) {
      const int ux = static_cast<int>(u % a.units_x), uy = static_cast<int>(u / a.units_x);
      int w_ok = 1;
      if (lane == 0) w_ok = ptx::mbar_wait(ptx::smem_u32(d_full), ucnt & 1u, abort_flag, lim) ? 1 : 0;
      w_ok = __shfl_sync(0xffffffffu, w_ok, 0);
      if (!w_ok) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
#pragma unroll 1
      for (int g = 0; g < 8; ++g) {  // 4 output channels at a time
        float m[16][4];
#pragma unroll
        for (int p = 0; p < 16; ++p) {
          uint32_t r[4];
          tmem_ld_x4(lane_base + p * 32 + 4 * g, r);
#pragma unroll
          for (int c = 0; c < 4; ++c) m[p][c] = __uint_as_float(r[c]);
        }
        ptx::tmem_wait_ld();
        float outv[2][2][4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          // fold the columns q first, then the rows p: Y = A^T M A
          float s0[4], s1[4];
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            s0[p] = m[4 * p + 0][c] + m[4 * p + 1][c] + m[4 * p + 2][c];
            s1[p] = m[4 * p + 1][c] - m[4 * p + 2][c] - m[4 * p + 3][c];
          }
          const float b = __ldg(a.bias + n0 + 4 * g + c);
          outv[0][0][c] = s0[0] + s0[1] + s0[2] + b;
          outv[0][1][c] = s1[0] + s1[1] + s1[2] + b;
          outv[1][0][c] = s0[1] - s0[2] - s0[3] + b;
          outv[1][1][c] = s1[1] - s1[2] - s1[3] + b;
        }
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            float v[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              v[c] = r16f(outv[i][j][c]);  // the Conv node's fp16 rounding
              if (a.act == kActRelu) v[c] = fmaxf(v[c], 0.f);
              else if (a.act == kActSilu) v[c] = r16f(v[c] * r16f(sigmoid_fast(v[c])));
            }
            const uint2 pk = make_uint2(h2u(__floats2half2_rn(v[0], v[1])), h2u(__floats2half2_rn(v[2], v[3])));
            *reinterpret_cast<uint2*>(stage + (i * 64 + 2 * lane + j) * kWStagePitch + g * 8) = pk;
          }
      }
      // All of this warp's accumulators are read: release them to the next unit's MMAs.
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(d_empty));
      // Residual adds and coalesced stores: 2 rows x 64 pixels x 4 chunks of 8 channels.
      const int xw = ux * kWUnitPx + 64 * (q & 1);
      const int yw = uy * kWUnitRows + 2 * tr;
#pragma unroll 4
      for (int idx = lane; idx < 2 * 64 * 4; idx += 32) {
        const int i = idx >> 8, px = (idx >> 2) & 63, ch = idx & 3;
        const int y = yw + i, x = xw + px;
        if (y >= a.H || x >= a.W) continue;
        uint4 v = *reinterpret_cast<const uint4*>(stage + (i * 64 + px) * kWStagePitch + ch * 16);
        const size_t off = (static_cast<size_t>(y) * a.W + x) * 64 + n0 + ch * 8;
        uint32_t* h = reinterpret_cast<uint32_t*>(&v);
        if (a.add1) {
          const uint4 r = __ldg(reinterpret_cast<const uint4*>(a.add1 + off));
          const uint32_t* rr = reinterpret_cast<const uint32_t*>(&r);
#pragma unroll
          for (int k = 0; k < 4; ++k) h[k] = h2u(__hadd2(u2h(h[k]), u2h(rr[k])));
        }
        if (a.add2) {
          const uint4 r = __ldg(reinterpret_cast<const uint4*>(a.add2 + off));
          const uint32_t* rr = reinterpret_cast<const uint32_t*>(&r);
#pragma unroll
          for (int k = 0; k < 4; ++k) h[k] = h2u(__hadd2(u2h(h[k]), u2h(rr[k])));
        }
        *reinterpret_cast<uint4*>(a.out + off) = v;
      }
      __syncwarp();
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, 512);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicOr(a.status, 1u);
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn wino_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

}  // namespace

bool wino_supported(int C, int M) { return C == 64 && M == 64; }

cudaError_t wino_upload(const uint16_t* w_oihw, const float* bias, int C, int M, WinoWeights* out) {
  if (!wino_supported(C, M)) return cudaErrorInvalidValue;
  // U = G g G^T per (m, c) in fp32, in the reference's summation order, then RNE to fp16
  // (src/vapoursynth/hip_engine.cc:972-1000); packed per (output half, point) as a
  // 32-row x 64-channel 128B-swizzled K-major block.
  static const float G[4][3] = {{1.f, 0.f, 0.f}, {.5f, .5f, .5f}, {.5f, -.5f, .5f}, {0.f, 0.f, 1.f}};
  std::vector<uint8_t> img(2 * kWUBytes, 0);
  for (int m = 0; m < M; ++m)
    for (int c = 0; c < C; ++c) {
      float g[9];
      for (int t = 0; t < 9; ++t) g[t] = HalfToFloat(w_oihw[(static_cast<size_t>(m) * C + c) * 9 + t]);
      float gg[4][3];
      for (int r = 0; r < 4; ++r)
        for (int cc = 0; cc < 3; ++cc) {
          float acc = 0.f;
          for (int k = 0; k < 3; ++k) acc += G[r][k] * g[k * 3 + cc];
          gg[r][cc] = acc;
        }
      for (int r = 0; r < 4; ++r)
        for (int cc = 0; cc < 4; ++cc) {
          float acc = 0.f;
          for (int k = 0; k < 3; ++k) acc += gg[r][k] * G[cc][k];
          const uint16_t h = FloatToHalfRNE(acc);
          const int p = r * 4 + cc, hn = m / 32, n = m % 32;
          uint8_t* blk = img.data() + static_cast<size_t>(hn) * kWUBytes + p * 4096;
          std::memcpy(blk + swz128(n, c / 8) + (c % 8) * 2, &h, 2);
        }
    }
  cudaError_t e = cudaMalloc(&out->upack, img.size());
  if (e != cudaSuccess) return e;
  e = cudaMemcpy(out->upack, img.data(), img.size(), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return e;
  std::vector<float> b(64, 0.f);
  if (bias) std::memcpy(b.data(), bias, sizeof(float) * M);
  e = cudaMalloc(&out->bias, sizeof(float) * 64);
  if (e != cudaSuccess) return e;
  return cudaMemcpy(out->bias, b.data(), sizeof(float) * 64, cudaMemcpyHostToDevice);
}

void wino_free(WinoWeights* w) {
  if (w->upack) cudaFree(w->upack);
  if (w->bias) cudaFree(w->bias);
  w->upack = nullptr;
  w->bias = nullptr;
}

bool wino_plan(const WinoWeights* w, const __half* in, int H, int W, __half* out, int num_sms, WinoPlan* P,
               std::string* err) {
  EncodeTiledFn enc = wino_encode_fn();
  if (!enc) {
    if (err) *err = "cuTensorMapEncodeTiled is unavailable from the CUDA driver";
    return false;
  }
  if ((reinterpret_cast<uintptr_t>(in) & 15u) || (reinterpret_cast<uintptr_t>(out) & 15u)) {
    if (err) *err = "Winograd conv buffers must be 16-byte aligned";
    return false;
  }
  cuuint64_t gdim[3] = {64, static_cast<cuuint64_t>(W), static_cast<cuuint64_t>(H)};
  cuuint64_t gstride[2] = {64 * 2, static_cast<cuuint64_t>(W) * 64 * 2};
  cuuint32_t box[3] = {16, static_cast<cuuint32_t>(kWBoxPx), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(&P->in_map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(in), gdim, gstride, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    if (err) *err = "cuTensorMapEncodeTiled failed (code " + std::to_string(static_cast<int>(r)) + ")";
    return false;
  }
  P->w = w;
  P->H = H;
  P->W = W;
  P->out = out;
  P->units_x = (W + kWUnitPx - 1) / kWUnitPx;
  P->units = static_cast<long long>(P->units_x) * ((H + kWUnitRows - 1) / kWUnitRows);
  long long gx = std::max(1, num_sms / 2);
  if (gx > P->units) gx = P->units;
  P->grid_x = static_cast<int>(gx);
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(conv3x3_wino_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kWSmem);
  });
  if (attr_err != cudaSuccess) {
    if (err) *err = std::string("cudaFuncSetAttribute failed: ") + cudaGetErrorString(attr_err);
    return false;
  }
  return true;
}

cudaError_t wino_launch(const WinoPlan& P, const __half* add1, const __half* add2, int act, uint32_t* status,
                        cudaStream_t stream) {
  WinoArgs a;
  std::memset(&a, 0, sizeof(a));
  a.in_map = P.in_map;
  a.upack = static_cast<const uint8_t*>(P.w->upack);
  a.bias = P.w->bias;
  a.add1 = add1 ? add1 : add2;
  a.add2 = add1 ? add2 : nullptr;
  a.out = P.out;
  a.status = status;
  a.H = P.H;
  a.W = P.W;
  a.act = act;
  a.units_x = P.units_x;
  a.units = P.units;
  a.wait_limit_ns = 4000000000ull;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(P.grid_x, 2);
  cfg.blockDim = dim3(kWThreads);
  cfg.dynamicSmemBytes = kWSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, conv3x3_wino_kernel, a);
}

}  // namespace ah
