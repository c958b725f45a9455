// Device side of the tcgen05 implicit-GEMM 3x3 convolution (stride 1, SAME padding).
//
// Replaces the reference's gfx1100 Winograd WMMA kernel (src/common/hip_kernels.h:143-396)
// for every conv whose input channel count fits the tensor-core tiling (C % 16 == 0,
// C <= 128), and the narrow tail conv with its fused DepthToSpace / Clip / boundary
// cast (the reference's dts_kernel_2d / dts_kernel_in_f32, hip_kernels.h:553-616).
//
// GEMM view: one output row segment of 128 pixels is the MMA M dimension, the output
// channels (padded to 16) are N, and K = 9 taps x C input channels. fp16 operands from
// shared memory, fp32 accumulators in tensor memory (TMEM). A bias MMA (a constant ones
// column times the bias row) initialises each accumulator.
//
// Data movement:
//  * input: one TMA tiled load per (input row, channel chunk) brings 130 pixels
//    (the 128-pixel tile plus a 1-pixel halo each side; out-of-range pixels and rows are
//    zero-filled by the TMA unit, which is the conv's zero padding) into a ring of row
//    slots. Each staged row feeds three output rows (ky = 0,1,2); the three horizontal
//    taps (kx) read the same slot with the descriptor start moved by one pixel row.
//  * weights: resident in shared memory for the whole persistent kernel, packed on the
//    host in the swizzled K-major layout the MMA reads.
//  * accumulators: a ring of NACC tensor-memory accumulators; the epilogue warps drain
//    one while the MMA warp fills the next.
//  * epilogue (8 warps; two per TMEM lane quarter, each taking alternate 32-channel
//    groups): tcgen05.ld -> fp16 rounding (the conv node output) -> ReLU / SiLU -> up to
//    two residual adds (fp16 adds, as the ONNX Add nodes) -> output.
//
// Two MMA formulations:
//  * standard (conv3x3_tc_kernel): per output row, 9 taps x C/16 MMAs of 128 x MT x 16;
//  * vertical window (conv3x3_tc_vert2_kernel, Mpad = 16, 32, 64): an input row feeds
//    output rows j, j-1, j-2 through kernel rows ky = 0, 1, 2; the weights of a
//    (kx, chunk) block hold the three kernel rows stacked along N, and the three output
//    rows sit in consecutive chunks of a TMEM ring, so one MMA of N = 3M per
//    (kx, k-block) does all three. It runs two row pipelines per CTA (below).
// Three output forms (EPI): 0 = NHWC fp16 through a swizzled staging tile and TMA stores;
// 1 = 2x DepthToSpace (DCR) into NCHW with paired stores (upscaler tails); 2 = general
// per-element DepthToSpace / clip / fp32 / layout stores.
//
// Every variant is a separate instantiation (chunk geometry x formulation x EPI x ACT), so
// each kernel's code holds only its own path: runtime switches in the per-row loops and
// their code size cost more than the work they select.
//
// Warp roles of the standard kernel (320 threads): warp 0 = TMA producer, warp 1 = TMEM
// allocator + MMA issuer (one thread), warps 2..9 = epilogue. Work: the (strip, row) space is split into
// contiguous ranges, one per CTA; every pipeline wait is time-bounded.
#pragma once

#include <cstdint>

#include "kernels.h"
#include "ptx.cuh"

namespace ah {
namespace tck {

constexpr int kMaxSlots = 8;
constexpr int kMaxAcc = 16;         // accumulator ring entries (16 = vertical mode, Mpad <= 32)
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kSmemLimit = 232448;  // 227 KB opt-in dynamic shared memory per block
constexpr int kStageTile = 2048;    // one 32-pixel x 32-channel fp16 staging tile
constexpr int kTailBytes = 1024;    // barriers and flags
constexpr int kSmemPerSm = 233472;  // shared memory of one SM (two CTAs share it)
constexpr int kVariants = 7;        // EPI 0 x ACT {none, relu, silu}; EPI 1; EPI 2; SiLU wide; EPI 3

struct ConvTcArgs {
  CUtensorMap maps[kTcMaxChunks];
  CUtensorMap out_map32;
  CUtensorMap out_map16;
  // Maps over the first loaded residual operand with the output tiles' geometry (used when
  // res_tma is set: the two-pipeline kernel then TMA-loads that operand into the staging
  // tiles one row ahead instead of loading it per lane).
  CUtensorMap res_map32;
  CUtensorMap res_map16;
  const uint8_t* wpack;
  const float* bias;
  const __half* add1;
  const __half* add2;
  uint32_t* status;
  ConvTcOut out;
  long long gofs[9 * kTcMaxChunks];
  int wofs[9 * kTcMaxChunks];
  int H, W, M, Mpad, MT;
  int c0[kTcMaxChunks];
  int slot_off[kTcMaxChunks];
  int slot_bytes;
  int slot_tx;  // bytes one row load delivers (all chunks, full boxes)
  int nslots;
  int w_smem_bytes;
  int ones_off, biasb_off, stage_off, stage_per_warp;
  long long rows_total;
  int act;
  int nacc, acc_stride;
  uint32_t tmem_cols;
  unsigned long long wait_limit_ns;  // bound of every pipeline wait (4 s)
  // Failure-path test hook (-1 = off): the producer arms this CTA-relative input row's
  // slot without loading it, so the MMA issuer's bounded wait for it runs out and the
  // kernel reports a timed-out wait in the status word instead of hanging.
  int stall_row;
  // Output form 0 only: the output buffer already holds the layer's last residual operand,
  // and the tile stores are TMA reduce-adds onto it (that operand is then not loaded).
  int reduce_out;
  int res_tma;
};

typedef void (*KernelFn)(ConvTcArgs);

// The instantiation for an input channel count (C % 16 == 0, 16 <= C <= 128), a
// formulation (vertical window, or standard) and an output variant (0-2: NHWC with act
// none/relu/silu, 3: 2x DepthToSpace tail, 4: general per-element output; vertical window
// only: 5 = 2 with eight epilogue warps per pipe, 640 threads; 6 = the kx-in-N 2x
// DepthToSpace tail of four conv channels).
KernelFn kernel_for(int C, bool vert, int variant);

struct Segment {
  int strip, ya, yb;
};

// Iterates the CTA's contiguous range of (strip, row) tiles as per-strip segments.
struct SegIter {
  long long t, t1;
  int H;
  __device__ __forceinline__ bool next(Segment& s) {
    if (t >= t1) return false;
    s.strip = static_cast<int>(t / H);
    s.ya = static_cast<int>(t % H);
    const long long left = t1 - t;
    s.yb = static_cast<int>(min(static_cast<long long>(H), s.ya + left));
    t = static_cast<long long>(s.strip) * H + s.yb;
    return true;
  }
};

__device__ __forceinline__ float r16(float v) { return __half2float(__float2half_rn(v)); }

// Position in a ring of S slots with its phase bit, advanced one step at a time (no integer
// division in the pipeline loops).
struct RingPos {
  uint32_t slot = 0, phase = 0;
  __device__ __forceinline__ void step(uint32_t S) {
    if (++slot == S) {
      slot = 0;
      phase ^= 1u;
    }
  }
};

// Byte offset of 16-byte granule j of row r in a swizzled K-major tile with `rb`-byte rows
// (128B / 64B / 32B swizzle: the granule index is XORed with address bits 7.. of the row,
// for a tile that starts on a 1024-byte boundary).
__host__ __device__ __forceinline__ uint32_t swz_granule(uint32_t r, uint32_t j, uint32_t rb) {
  const uint32_t phase = rb == 128 ? (r & 7u) : (rb == 64 ? ((r >> 1) & 3u) : ((r >> 2) & 1u));
  return r * rb + ((j ^ phase) << 4);
}

__device__ __forceinline__ void hadd8v(uint32_t (&h)[4], const uint4& u) {
  const uint32_t* q = reinterpret_cast<const uint32_t*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 v = __hadd2(*reinterpret_cast<__half2*>(&h[i]), *reinterpret_cast<const __half2*>(&q[i]));
    h[i] = *reinterpret_cast<uint32_t*>(&v);
  }
}

// Activation on 8 channels held as 4 half2 (the fp16-rounded conv output).
template <int ACT>
__device__ __forceinline__ void act8(uint32_t (&h)[4]) {
  if constexpr (ACT == kActSilu) {
    // Sigmoid rounded to fp16, then the fp16 product: the fp32 product of two fp16 values
    // is exact, so one rounded half2 multiply equals rounding it (the graph's Mul node).
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __half2 v = *reinterpret_cast<__half2*>(&h[i]);
      const float2 t = __half22float2(v);
      const __half2 sg = __floats2half2_rn(sigmoid_fast(t.x), sigmoid_fast(t.y));
      __half2 o = __hmul2(v, sg);
      h[i] = *reinterpret_cast<uint32_t*>(&o);
    }
  } else if constexpr (ACT == kActRelu) {
    const __half2 z = __float2half2_rn(0.f);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 v = __hmax2(*reinterpret_cast<__half2*>(&h[i]), z);
      h[i] = *reinterpret_cast<uint32_t*>(&v);
    }
  }
}

// Activation of one fp16-rounded conv output value (runtime selector).
__device__ __forceinline__ float act1(float t, int act) {
  if (act == kActRelu) return fmaxf(t, 0.f);
  if (act == kActSilu) return r16(t * r16(sigmoid_fast(t)));
  return t;
}

// Narrow tail with a fused 2x DepthToSpace (DCR) into an NCHW output, M = 4 * COUT channels
// all in this thread's accumulator row: output channel c, sub-row r of pixel x takes conv
// channels (2r)*COUT + c and (2r+1)*COUT + c, which land side by side in the output row, so
// each (c, r) is one 4-byte (fp16) or 8-byte (fp32) store and a warp writes 128 / 256
// contiguous bytes per store instruction.
template <int COUT>
__device__ __forceinline__ void store_dts2_nchw(const uint32_t (&rr)[32], int act, const ConvTcOut& o, int y, int x,
                                                int H, int W) {
  const long long Wo = 2LL * W, plane = 4LL * H * W;
  const long long row0 = 2LL * y * Wo + 2LL * x;
#pragma unroll
  for (int c = 0; c < COUT; ++c)
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float t[2];
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        float v = act1(r16(__uint_as_float(rr[(2 * r + q) * COUT + c])), act);
        if (o.clip) v = fminf(fmaxf(v, o.clip_lo), o.clip_hi);
        t[q] = v;
      }
      const long long idx = c * plane + row0 + r * Wo;
      if (o.fp32) *reinterpret_cast<float2*>(static_cast<float*>(o.ptr) + idx) = make_float2(t[0], t[1]);
      else *reinterpret_cast<__half2*>(static_cast<__half*>(o.ptr) + idx) = __floats2half2_rn(t[0], t[1]);
    }
}

// Compile-time geometry of the input-channel chunks (64-channel chunks first, then at most
// one 32 and one 16, matching the host's chunking). The MMA issue loop is fully unrolled
// over it, so every descriptor is a register plus a constant: a single issuing thread
// keeps the tensor core fed (runtime-computed descriptors cost 77-120 cycles per MMA on
// B200, above the 48-cycle execution time of a 128x64x16 MMA).
template <int NC64, int NC32, int NC16>
struct ChunkCfg {
  static constexpr int N = NC64 + NC32 + NC16;
  static constexpr int C = 64 * NC64 + 32 * NC32 + 16 * NC16;
  __host__ __device__ static constexpr int rb(int k) { return k < NC64 ? 128 : (k < NC64 + NC32 ? 64 : 32); }
  __host__ __device__ static constexpr int kblocks(int k) { return rb(k) / 32; }
  __host__ __device__ static constexpr uint32_t layout(int k) { return rb(k) == 128 ? 2u : (rb(k) == 64 ? 4u : 6u); }
  __host__ __device__ static constexpr int area(int k) { return (136 * rb(k) + 1023) / 1024 * 1024; }
  __host__ __device__ static constexpr int off(int k) { return k == 0 ? 0 : off(k - 1) + area(k - 1); }
  // Slot layout of the kx-in-N tail: four 32-pixel sub-tiles (128 rows) per chunk.
  __host__ __device__ static constexpr int off128(int k) { return k == 0 ? 0 : off128(k - 1) + 128 * rb(k - 1); }
  __host__ __device__ static constexpr uint32_t hi(int k) { return ptx::desc_hi(8u * rb(k), layout(k)); }
};

// The MMAs of one input row in the vertical-window formulation: for every (chunk, kx,
// k-block) one MMA of N = n1 * M into the window's first TMEM run and, where the window
// wraps around the accumulator ring (SPLIT), a second one into the run at column 0.
// NKX = 1 is the kx-in-N tail: one weight block per chunk holds all three kx, and the A
// operand is the slot's 128 rows (four 32-pixel sub-tiles).
template <class Cfg, bool SPLIT, int NKX = 3>
__device__ __forceinline__ void vert_row_mmas(uint32_t sl, const uint32_t (&bv)[3][Cfg::N], uint32_t M,
                                              uint32_t ky_lo, uint32_t n1, uint32_t d1, uint32_t d2, uint32_t i1,
                                              uint32_t i2) {
#pragma unroll
  for (int k = 0; k < Cfg::N; ++k) {
    const uint32_t mrows16 = (M * Cfg::rb(k)) >> 4;  // M weight rows, in 16-byte units
    const uint32_t b1 = ky_lo * mrows16, b2 = (ky_lo + n1) * mrows16;
#pragma unroll
    for (int kx = 0; kx < NKX; ++kx)
#pragma unroll
      for (int kb = 0; kb < Cfg::kblocks(k); ++kb) {
        const uint32_t alo = sl + (((NKX == 1 ? Cfg::off128(k) : Cfg::off(k)) + kx * Cfg::rb(k) + kb * 32) >> 4);
        const uint32_t blo = bv[kx][k] + kb * 2;
        ptx::mma_f16_ss_acc(d1, alo, Cfg::hi(k), blo + b1, Cfg::hi(k), i1);
        if (SPLIT) ptx::mma_f16_ss_acc(d2, alo, Cfg::hi(k), blo + b2, Cfg::hi(k), i2);
      }
  }
}

template <int NC64, int NC32, int NC16, int EPI, int ACT>
__global__ void __launch_bounds__(kThreads, 1) conv3x3_tc_kernel(const __grid_constant__ ConvTcArgs a) {
  using Cfg = ChunkCfg<NC64, NC32, NC16>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sW = smem;
  uint8_t* sA = smem + a.w_smem_bytes;
  uint8_t* sOnes = smem + a.ones_off;
  uint8_t* sBiasB = smem + a.biasb_off;
  uint8_t* sStage = smem + a.stage_off;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sStage + kEpiWarps * a.stage_per_warp);
  uint64_t* full = bars;
  uint64_t* empty = bars + kMaxSlots;
  uint64_t* accf = bars + 2 * kMaxSlots;
  uint64_t* acce = accf + kMaxAcc;
  uint64_t* wbar = acce + kMaxAcc;
  uint64_t* donebar = wbar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(donebar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * a.MT;
  ptx::griddep_launch_dependents();  // the next layer's CTAs may take SMs this grid frees
  const int S = a.nslots;
  const int NACC = a.nacc;  // a power of two
  const uint32_t lgA = 31 - __clz(static_cast<uint32_t>(NACC));

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(ptx::smem_u32(&full[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&empty[s]), 1);
    }
    for (int i = 0; i < NACC; ++i) {
      ptx::mbar_init(ptx::smem_u32(&accf[i]), 1);
      ptx::mbar_init(ptx::smem_u32(&acce[i]), kEpiWarps);
    }
    ptx::mbar_init(ptx::smem_u32(wbar), 1);
    ptx::mbar_init(ptx::smem_u32(donebar), 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
#pragma unroll
    for (int k = 0; k < Cfg::N; ++k) ptx::prefetch_tensormap(&a.maps[k]);
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_u32(tmem_slot), a.tmem_cols);
    ptx::tmem_relinquish();
  }
  // Bias operands (32-byte swizzled rows, 16 K elements): a ones column for the 128
  // pixel rows, and the bias as column 0 of the MT output-channel rows.
  for (int r = threadIdx.x; r < kTcTilePx; r += blockDim.x) {
    uint4* row = reinterpret_cast<uint4*>(sOnes + r * 32);
    row[0] = make_uint4(0, 0, 0, 0);
    row[1] = make_uint4(0, 0, 0, 0);
    *reinterpret_cast<__half*>(sOnes + swz_granule(r, 0, 32)) = __float2half(1.f);
  }
  for (int r = threadIdx.x; r < a.MT; r += blockDim.x) {
    uint4* row = reinterpret_cast<uint4*>(sBiasB + r * 32);
    row[0] = make_uint4(0, 0, 0, 0);
    row[1] = make_uint4(0, 0, 0, 0);
    *reinterpret_cast<__half*>(sBiasB + swz_granule(r, 0, 32)) = __float2half(a.bias[m0 + r]);
  }
  ptx::fence_proxy_async_smem();  // the tensor core reads the generic writes above
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const long long t0 = static_cast<long long>(blockIdx.x) * a.rows_total / gridDim.x;
  const long long t1 = static_cast<long long>(blockIdx.x + 1) * a.rows_total / gridDim.x;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      // weight blocks: 9 taps x chunks of MT rows
      constexpr int nblk = 9 * Cfg::N;
      const int wrows = a.MT;
      uint32_t wbytes = 0;
#pragma unroll
      for (int idx = 0; idx < nblk; ++idx) wbytes += wrows * Cfg::rb(idx % Cfg::N);
      ptx::mbar_arrive_expect_tx(ptx::smem_u32(wbar), wbytes);
#pragma unroll
      for (int idx = 0; idx < nblk; ++idx) {
        const int k = idx % Cfg::N;
        const uint8_t* src = a.wpack + a.gofs[idx] + static_cast<long long>(m0) * Cfg::rb(k);
        ptx::bulk_load(ptx::smem_u32(sW + a.wofs[idx]), src, wrows * Cfg::rb(k), ptx::smem_u32(wbar));
      }
      ptx::griddep_wait();  // the input rows come from the previous layer
      uint32_t g = 0;
      RingPos rp;
      SegIter it{t0, t1, a.H};
      Segment sg;
      bool ok = true;
      while (ok && it.next(sg)) {
        const int x0 = sg.strip * kTcTilePx - 1;
        for (int r = sg.ya - 1; r <= sg.yb; ++r, ++g, rp.step(S)) {
          const uint32_t slot = rp.slot;
          if (!ptx::mbar_wait(ptx::smem_u32(&empty[slot]), rp.phase ^ 1u, abort_flag, a.wait_limit_ns)) {
            ok = false;
            break;
          }
          const uint32_t fb = ptx::smem_u32(&full[slot]);
          ptx::mbar_arrive_expect_tx(fb, a.slot_tx);
          if (static_cast<int>(g) == a.stall_row) continue;  // failure-path test: never completes
          const uint32_t dst = ptx::smem_u32(sA + slot * a.slot_bytes);
#pragma unroll
          for (int k = 0; k < Cfg::N; ++k) ptx::tma_load_3d(dst + Cfg::off(k), &a.maps[k], fb, a.c0[k], x0, r);
        }
      }
      // Never leave a TMA write in flight at exit: wait (time-bounded) for the last loads.
      volatile int never_abort = 0;
      const uint32_t first = g > static_cast<uint32_t>(S) ? g - S : 0u;
      for (uint32_t j = first; j < g; ++j)
        ptx::mbar_wait(ptx::smem_u32(&full[j % S]), (j / S) & 1u, &never_abort, a.wait_limit_ns);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t sA_u = ptx::smem_u32(sA);
      const uint32_t sW_u = ptx::smem_u32(sW);
      const uint64_t ones_desc = ptx::smem_desc(ptx::smem_u32(sOnes), 6, 256);
      const uint64_t biasb_desc = ptx::smem_desc(ptx::smem_u32(sBiasB), 6, 256);
      const uint32_t alo0 = ptx::desc_lo(sA_u);
      const uint32_t slot16 = static_cast<uint32_t>(a.slot_bytes) >> 4;
      bool ok = ptx::mbar_wait(ptx::smem_u32(wbar), 0, abort_flag, a.wait_limit_ns);
      SegIter it{t0, t1, a.H};
      Segment sg;
      const uint32_t idesc = ptx::idesc_f16_f32(kTcTilePx, a.MT);
      uint32_t blo[9][Cfg::N];
#pragma unroll
      for (int t = 0; t < 9; ++t)
#pragma unroll
        for (int k = 0; k < Cfg::N; ++k) blo[t][k] = ptx::desc_lo(sW_u + a.wofs[t * Cfg::N + k]);
      uint32_t acc_cnt = 0;
      RingPos rp;  // ring position of the next input row to wait for
      while (ok && it.next(sg)) {
        const int n = sg.yb - sg.ya;
        uint32_t slot[3];
        for (int ky = 0; ky < 2 && ok; ++ky, rp.step(S)) {  // the first two rows of the segment
          slot[ky] = rp.slot;
          ok = ptx::mbar_wait(ptx::smem_u32(&full[slot[ky]]), rp.phase, abort_flag, a.wait_limit_ns);
        }
        for (int i = 0; i < n && ok; ++i) {
          // rows i and i+1 of the segment were waited for already; wait for row i+2
          slot[2] = rp.slot;
          ok = ptx::mbar_wait(ptx::smem_u32(&full[slot[2]]), rp.phase, abort_flag, a.wait_limit_ns);
          rp.step(S);
          const uint32_t acc = acc_cnt & (NACC - 1);
          if (ok) ok = ptx::mbar_wait(ptx::smem_u32(&acce[acc]), ((acc_cnt >> lgA) & 1u) ^ 1u, abort_flag, a.wait_limit_ns);
          if (!ok) break;
          ptx::tc_fence_after();
          const uint32_t d = tmem_base + acc * a.acc_stride;
          ptx::mma_f16_ss(d, ones_desc, biasb_desc, idesc, 0);  // D = bias
#pragma unroll
          for (int ky = 0; ky < 3; ++ky) {
            const uint32_t sl = alo0 + slot[ky] * slot16;
#pragma unroll
            for (int k = 0; k < Cfg::N; ++k)
#pragma unroll
              for (int kx = 0; kx < 3; ++kx)
#pragma unroll
                for (int kb = 0; kb < Cfg::kblocks(k); ++kb)
                  ptx::mma_f16_ss_acc(d, sl + ((Cfg::off(k) + kx * Cfg::rb(k) + kb * 32) >> 4), Cfg::hi(k),
                                      blo[ky * 3 + kx][k] + kb * 2, Cfg::hi(k), idesc);
          }
          ptx::mma_commit(ptx::smem_u32(&accf[acc]));
          ptx::mma_commit(ptx::smem_u32(&empty[slot[0]]));
          slot[0] = slot[1];
          slot[1] = slot[2];
          ++acc_cnt;
        }
        if (!ok) break;
        ptx::mma_commit(ptx::smem_u32(&empty[slot[0]]));  // the segment's last two rows
        ptx::mma_commit(ptx::smem_u32(&empty[slot[1]]));
      }
      // Drain every issued MMA before the tensor memory is released.
      ptx::mma_commit(ptx::smem_u32(donebar));
      volatile int never_abort = 0;
      ptx::mbar_wait(ptx::smem_u32(donebar), 0, &never_abort, a.wait_limit_ns);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (warps 2..9) ----------------
    ptx::griddep_wait();  // residual operands and the output buffer belong to earlier layers
    const int e = warp - 2;
    const int q = warp & 3;   // tensor-memory lane quarter this warp may access
    const int half = e >> 2;  // this warp takes channel groups half, half+2, ...
    const int ngroups = (a.MT + 31) / 32;
    const int act = ACT >= 0 ? ACT : a.act;
    uint8_t* stage = sStage + e * a.stage_per_warp;
    const ConvTcOut& o = a.out;
    uint32_t acc_cnt = 0;
    SegIter it{t0, t1, a.H};
    Segment sg;
    bool ok = true;
    bool stores_pending = false;
    while (ok && it.next(sg)) {
      const int xw = sg.strip * kTcTilePx + q * 32;  // first pixel of this warp's 32
      const int x = xw + lane;
      const bool valid = x < a.W;
      for (int y = sg.ya; y < sg.yb; ++y) {
        const uint32_t acc = acc_cnt & (NACC - 1);  // accumulator of this output row
        const size_t pix = static_cast<size_t>(y) * a.W + (valid ? x : 0);
        if constexpr (EPI == 0) {
          // Residual lines of the row two ahead go to L2 now, so the register loads below
          // (issued one accumulator wait ahead) hit L2 instead of DRAM.
          if (valid && a.add1 && half < ngroups && y + 2 < sg.yb) {
            const size_t off = (pix + 2 * static_cast<size_t>(a.W)) * a.M + m0 + half * 32;
            ptx::prefetch_l2(a.add1 + off);
            if (a.add2) ptx::prefetch_l2(a.add2 + off);
          }
        }
        // Residual operands of this warp's first two channel groups, loaded before the
        // accumulator wait so their DRAM latency overlaps the row's MMAs.
        uint4 pre[2][2][4];
        if constexpr (EPI == 0) {
          if (valid && a.add1) {
#pragma unroll
            for (int k = 0; k < 2; ++k) {
              const int g = half + 2 * k;
              if (g >= ngroups) break;
              const int cw = min(32, a.MT - g * 32);
              const size_t off = pix * a.M + m0 + g * 32;
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                if (i * 8 >= cw) break;
                pre[0][k][i] = __ldg(reinterpret_cast<const uint4*>(a.add1 + off + i * 8));
                if (a.add2) pre[1][k][i] = __ldg(reinterpret_cast<const uint4*>(a.add2 + off + i * 8));
              }
            }
          }
        }
        int w_ok = 0;
        if (lane == 0) w_ok = ptx::mbar_wait(ptx::smem_u32(&accf[acc]), (acc_cnt >> lgA) & 1u, abort_flag, a.wait_limit_ns) ? 1 : 0;
        w_ok = __shfl_sync(0xffffffffu, w_ok, 0);
        if (!w_ok) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        if constexpr (EPI == 0) {
          if (stores_pending) {
            if (lane == 0) ptx::bulk_wait_group_read0();  // the staging tiles are free again
            __syncwarp();
          }
        }
        if (half >= ngroups) {  // no channel group for this warp (MT <= 32): just release
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(&acce[acc]));
        }
        // At most 4 groups per warp (MT <= 256); unrolled so the prefetched operands of
        // groups 0 and 1 stay in registers.
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int g = half + 2 * k;
          if (g >= ngroups) break;
          const int cw = min(32, a.MT - g * 32);
          uint32_t rr[32];
          const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * a.acc_stride + g * 32;
          if (cw == 32) ptx::tmem_ld_32x32b_x32(taddr, rr);
          else ptx::tmem_ld_32x32b_x16(taddr, rr);
          ptx::tmem_wait_ld();
          if (g + 2 >= ngroups) {  // this warp's last group: release the accumulator
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(&acce[acc]));
          }
          const int cbase = m0 + g * 32;
          if constexpr (EPI == 0) {
            uint8_t* st = stage + k * kStageTile;
            const uint32_t rb = cw * 2;
#pragma unroll
            for (int j8 = 0; j8 < 32; j8 += 8) {
              if (j8 >= cw) break;
              uint32_t h[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                __half2 v = __floats2half2_rn(__uint_as_float(rr[j8 + 2 * i]), __uint_as_float(rr[j8 + 2 * i + 1]));
                h[i] = *reinterpret_cast<uint32_t*>(&v);
              }
              act8<ACT>(h);
              if (valid && a.add1) {
                if (k < 2) {
                  hadd8v(h, pre[0][k][j8 >> 3]);
                  if (a.add2) hadd8v(h, pre[1][k][j8 >> 3]);
                } else {
                  const size_t off = pix * a.M + cbase + j8;
                  hadd8v(h, __ldg(reinterpret_cast<const uint4*>(a.add1 + off)));
                  if (a.add2) hadd8v(h, __ldg(reinterpret_cast<const uint4*>(a.add2 + off)));
                }
              }
              *reinterpret_cast<uint4*>(st + swz_granule(lane, j8 >> 3, rb)) = make_uint4(h[0], h[1], h[2], h[3]);
            }
          } else if constexpr (EPI == 1) {
            if (valid) {
              switch (a.M >> 2) {
                case 1: store_dts2_nchw<1>(rr, act, o, y, x, a.H, a.W); break;
                case 2: store_dts2_nchw<2>(rr, act, o, y, x, a.H, a.W); break;
                case 3: store_dts2_nchw<3>(rr, act, o, y, x, a.H, a.W); break;
                default: store_dts2_nchw<4>(rr, act, o, y, x, a.H, a.W); break;
              }
            }
          } else {
            if (valid) {
              // General narrow outputs: per-element DepthToSpace (DCR) / clip / dtype / layout.
              const int b = o.dts_b;
              const int cout = a.M / (b * b);
              const long long Ho = static_cast<long long>(a.H) * b, Wo = static_cast<long long>(a.W) * b;
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const int m = cbase + j;
                if (j >= cw || m >= a.M) break;
                float t = act1(r16(__uint_as_float(rr[j])), act);
                if (a.add1) t = r16(t + __half2float(a.add1[pix * a.M + m]));
                if (a.add2) t = r16(t + __half2float(a.add2[pix * a.M + m]));
                if (o.clip) t = fminf(fmaxf(t, o.clip_lo), o.clip_hi);
                const int rq = m / cout, c = m - rq * cout;
                const int r_ = rq / b, q_ = rq - r_ * b;
                const long long oy = static_cast<long long>(y) * b + r_, ox = static_cast<long long>(x) * b + q_;
                const long long idx =
                    o.nchw ? ((static_cast<long long>(c) * Ho + oy) * Wo + ox) : ((oy * Wo + ox) * cout + c);
                if (o.fp32) static_cast<float*>(o.ptr)[idx] = t;
                else static_cast<__half*>(o.ptr)[idx] = __float2half_rn(t);
              }
            }
          }
        }
        if constexpr (EPI == 0) {
          ptx::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && xw < a.W) {
            for (int g = half, k = 0; g < ngroups; g += 2, ++k) {
              const int cw = min(32, a.MT - g * 32);
              const uint32_t src = ptx::smem_u32(stage + k * kStageTile);
              const CUtensorMap* map = cw == 32 ? &a.out_map32 : &a.out_map16;
              if (a.reduce_out) ptx::tma_reduce_add_3d(map, src, m0 + g * 32, xw, y);
              else ptx::tma_store_3d(map, src, m0 + g * 32, xw, y);
            }
            ptx::bulk_commit_group();
          }
          stores_pending = true;
        }
        ++acc_cnt;
      }
    }
    if constexpr (EPI == 0) {
      if (lane == 0) ptx::bulk_wait_group0();
    }
    __syncwarp();
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, a.tmem_cols);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicOr(a.status, 1u);
}

// ---------------------------------------------------------------------------
// Vertical-window formulation with two row pipelines per CTA (384 threads). A single
// MMA-issuing thread spends ~750 cycles per input row on waits, commits and loop control
// between its ~1,050 cycles of MMAs, and the tensor core idles meanwhile. Two issuers,
// each running its own half of the CTA's rows with its own input-slot ring, TMEM ring
// (half of the 512 columns) and four epilogue warps, keep it busy while sharing one copy
// of the weights in shared memory.
//
// Warps: 0 and 3 = TMA producers (pipe 0 / 1; warp 0 also loads the weights), 1 and 2 =
// MMA issuers (pipe 0 / 1; warp 1 allocates TMEM), 4..7 = epilogue of pipe 0 and 8..11 =
// epilogue of pipe 1 (warp w reads TMEM lane quarter w % 4 and all channel groups). With
// WIDE (640 threads), 4..11 and 12..19 are the pipes' epilogues, warp w taking lane quarter
// w % 4 and 32-channel group ((w - 4) / 4) % 2. The 2x DepthToSpace tail (EPI 1) is built
// for two CTAs per SM, each with half of the TMEM columns.
//
// kx-in-N tail (EPI 3, M = 4 output channels before a 2x DepthToSpace): the three
// horizontal taps move from K into N. One weight block per chunk holds, per kernel row ky,
// the 16 columns kx * 4 + m (12 used), so an input row takes C / 16 MMAs of N = 48 instead
// of 3 * C / 16. TMEM lane l then holds the three partial sums P_kx (bias on kx = 1) of
// the pixel in slot row l, and an output pixel p takes P_0(p - 1) + P_1(p) + P_2(p + 1).
// The slot holds four 32-pixel sub-tiles loaded 30 pixels apart (one TMA load each), so
// the 32 lanes a warp may read (TMEM lane quarter q) cover pixels x0 + 30q - 1 .. +30:
// lanes 1..30 output, their neighbours come by warp shuffle, and no warp waits for
// another. A strip advances 120 pixels.
// ---------------------------------------------------------------------------
constexpr int kThreads2 = 384;
// Wide epilogue (SiLU NHWC layers of 64 channels, whose epilogue math is the bound): eight
// epilogue warps per pipe, one per (TMEM lane quarter, 32-channel group).
constexpr int kThreads2W = 640;
constexpr int kMaxEpiWarps2 = 16;
// kx-in-N tail: pixels per sub-tile load, pixels a sub-tile advances (30 outputs per
// warp), and pixels a strip advances.
constexpr int kKxnSub = 32;
constexpr int kKxnSubStep = 30;
constexpr int kKxnStride = 4 * kKxnSubStep;

template <int NC64, int NC32, int NC16, int EPI, int ACT, int WIDE>
__global__ void __launch_bounds__(WIDE ? kThreads2W : kThreads2, (EPI == 1 || EPI == 3) ? 2 : 1)
    conv3x3_tc_vert2_kernel(const __grid_constant__ ConvTcArgs a) {
  using Cfg = ChunkCfg<NC64, NC32, NC16>;
  static_assert(!WIDE || EPI == 0, "the wide epilogue is for NHWC outputs");
  constexpr int kStride = EPI == 3 ? kKxnStride : kTcTilePx;  // pixels a strip advances
  constexpr int NKX = EPI == 3 ? 1 : 3;                        // weight blocks (kx) per chunk
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sW = smem;
  uint8_t* sA = smem + a.w_smem_bytes;  // pipe p, slot s at sA + (p * S + s) * slot_bytes
  uint8_t* sOnes = smem + a.ones_off;
  uint8_t* sBiasB = smem + a.biasb_off;
  uint8_t* sStage = smem + a.stage_off;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sStage + 8 * a.stage_per_warp);
  uint64_t* full = bars;                       // [2][kMaxSlots]
  uint64_t* empty = full + 2 * kMaxSlots;      // [2][kMaxSlots]
  uint64_t* accf = empty + 2 * kMaxSlots;      // [2][kMaxAcc]
  uint64_t* acce = accf + 2 * kMaxAcc;         // [2][kMaxAcc]
  uint64_t* wbar = acce + 2 * kMaxAcc;
  uint64_t* donebar = wbar + 1;                // [2]
  uint64_t* rbar = donebar + 2;                // [kMaxEpiWarps2] residual tiles of the epilogue warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + kMaxEpiWarps2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  ptx::griddep_launch_dependents();  // the next layer's CTAs may take SMs this grid frees
  const int S = a.nslots;           // input-row slots per pipe
  const int NACC = a.nacc;          // accumulator chunks per pipe (a power of two)
  const uint32_t lgA = 31 - __clz(static_cast<uint32_t>(NACC));
  const uint32_t M = a.MT;          // = Mpad: one chunk of M columns per output row
  const uint32_t half_cols = a.tmem_cols / 2;
  const int m0 = blockIdx.y * a.MT;  // this CTA's slice of output channels

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2 * S; ++i) {
      const int pp = i / S, ss = i - pp * S;
      ptx::mbar_init(ptx::smem_u32(&full[pp * kMaxSlots + ss]), 1);
      ptx::mbar_init(ptx::smem_u32(&empty[pp * kMaxSlots + ss]), 1);
    }
    for (int i = 0; i < 2 * NACC; ++i) {
      const int pp = i / NACC, cc = i - pp * NACC;
      ptx::mbar_init(ptx::smem_u32(&accf[pp * kMaxAcc + cc]), 1);
      ptx::mbar_init(ptx::smem_u32(&acce[pp * kMaxAcc + cc]), WIDE ? 8 : 4);  // the pipe's epilogue warps
    }
    ptx::mbar_init(ptx::smem_u32(wbar), 1);
    ptx::mbar_init(ptx::smem_u32(&donebar[0]), 1);
    ptx::mbar_init(ptx::smem_u32(&donebar[1]), 1);
    for (int i = 0; i < kMaxEpiWarps2; ++i) ptx::mbar_init(ptx::smem_u32(&rbar[i]), 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if ((warp == 0 || warp == 3) && lane == 0) {
#pragma unroll
    for (int k = 0; k < Cfg::N; ++k) ptx::prefetch_tensormap(&a.maps[k]);
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_u32(tmem_slot), a.tmem_cols);
    ptx::tmem_relinquish();
  }
  // Bias operands (32-byte swizzled rows, 16 K elements): a ones column for the 128
  // pixel rows, and the bias as column 0 of the M output-channel rows.
  for (int r = threadIdx.x; r < kTcTilePx; r += blockDim.x) {
    uint4* row = reinterpret_cast<uint4*>(sOnes + r * 32);
    row[0] = make_uint4(0, 0, 0, 0);
    row[1] = make_uint4(0, 0, 0, 0);
    *reinterpret_cast<__half*>(sOnes + swz_granule(r, 0, 32)) = __float2half(1.f);
  }
  for (int r = threadIdx.x; r < a.MT; r += blockDim.x) {
    uint4* row = reinterpret_cast<uint4*>(sBiasB + r * 32);
    row[0] = make_uint4(0, 0, 0, 0);
    row[1] = make_uint4(0, 0, 0, 0);
    float bv = 0.f;
    if constexpr (EPI == 3) {  // columns kx * M + m: the bias goes with the centre tap kx = 1
      if (r >= a.M && r < 2 * a.M) bv = a.bias[r - a.M];
    } else {
      bv = a.bias[m0 + r];
    }
    *reinterpret_cast<__half*>(sBiasB + swz_granule(r, 0, 32)) = __float2half(bv);
  }
  ptx::fence_proxy_async_smem();  // the tensor core reads the generic writes above
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // The CTA's contiguous (strip, row) range, split between the two pipes.
  const long long t0 = static_cast<long long>(blockIdx.x) * a.rows_total / gridDim.x;
  const long long t1 = static_cast<long long>(blockIdx.x + 1) * a.rows_total / gridDim.x;
  const long long tm = (t0 + t1) / 2;

  if (warp == 0 || warp == 3) {
    // ---------------- TMA producers ----------------
    const int pp = warp == 0 ? 0 : 1;
    if (lane == 0) {
      if (pp == 0) {
        // weight blocks: 3 kx x chunks of 3M rows (the three ky stacked); EPI 3: one block
        // per chunk
        constexpr int nblk = NKX * Cfg::N;
        const int wrows = 3 * a.MT;
        uint32_t wbytes = 0;
#pragma unroll
        for (int idx = 0; idx < nblk; ++idx) wbytes += wrows * Cfg::rb(idx % Cfg::N);
        ptx::mbar_arrive_expect_tx(ptx::smem_u32(wbar), wbytes);
#pragma unroll
        for (int idx = 0; idx < nblk; ++idx) {
          const int k = idx % Cfg::N;
          ptx::bulk_load(ptx::smem_u32(sW + a.wofs[idx]),
                         a.wpack + a.gofs[idx] + static_cast<long long>(3 * m0) * Cfg::rb(k), wrows * Cfg::rb(k),
                         ptx::smem_u32(wbar));
        }
      }
      ptx::griddep_wait();  // the input rows come from the previous layer
      uint64_t* pfull = full + pp * kMaxSlots;
      uint64_t* pempty = empty + pp * kMaxSlots;
      uint8_t* pA = sA + static_cast<size_t>(pp) * S * a.slot_bytes;
      uint32_t g = 0;
      RingPos rp;
      SegIter it{pp == 0 ? t0 : tm, pp == 0 ? tm : t1, a.H};
      Segment sg;
      bool ok = true;
      while (ok && it.next(sg)) {
        const int x0 = sg.strip * kStride - 1;
        for (int r = sg.ya - 1; r <= sg.yb; ++r, ++g, rp.step(S)) {
          const uint32_t slot = rp.slot;
          if (!ptx::mbar_wait(ptx::smem_u32(&pempty[slot]), rp.phase ^ 1u, abort_flag, a.wait_limit_ns)) {
            ok = false;
            break;
          }
          const uint32_t fb = ptx::smem_u32(&pfull[slot]);
          ptx::mbar_arrive_expect_tx(fb, a.slot_tx);
          if (static_cast<int>(g) == a.stall_row) continue;  // failure-path test: never completes
          const uint32_t dst = ptx::smem_u32(pA + slot * a.slot_bytes);
          if constexpr (EPI == 3) {
#pragma unroll
            for (int k = 0; k < Cfg::N; ++k)
#pragma unroll
              for (int sq = 0; sq < 4; ++sq)
                ptx::tma_load_3d(dst + Cfg::off128(k) + sq * kKxnSub * Cfg::rb(k), &a.maps[k], fb, a.c0[k],
                                 x0 + sq * kKxnSubStep, r);
          } else {
#pragma unroll
            for (int k = 0; k < Cfg::N; ++k) ptx::tma_load_3d(dst + Cfg::off(k), &a.maps[k], fb, a.c0[k], x0, r);
          }
        }
      }
      // Never leave a TMA write in flight at exit: wait (time-bounded) for the last loads.
      volatile int never_abort = 0;
      const uint32_t first = g > static_cast<uint32_t>(S) ? g - S : 0u;
      for (uint32_t j = first; j < g; ++j)
        ptx::mbar_wait(ptx::smem_u32(&pfull[j % S]), (j / S) & 1u, &never_abort, a.wait_limit_ns);
    }
  } else if (warp == 1 || warp == 2) {
    // ---------------- MMA issuers ----------------
    const int pp = warp - 1;
    if (lane == 0) {
      uint64_t* pfull = full + pp * kMaxSlots;
      uint64_t* pempty = empty + pp * kMaxSlots;
      uint64_t* paccf = accf + pp * kMaxAcc;
      uint64_t* pacce = acce + pp * kMaxAcc;
      const uint32_t tbase = tmem_base + pp * half_cols;
      const uint32_t sA_u = ptx::smem_u32(sA + static_cast<size_t>(pp) * S * a.slot_bytes);
      const uint32_t sW_u = ptx::smem_u32(sW);
      const uint64_t ones_desc = ptx::smem_desc(ptx::smem_u32(sOnes), 6, 256);
      const uint64_t biasb_desc = ptx::smem_desc(ptx::smem_u32(sBiasB), 6, 256);
      const uint32_t alo0 = ptx::desc_lo(sA_u);
      const uint32_t slot16 = static_cast<uint32_t>(a.slot_bytes) >> 4;
      const uint32_t NCH = NACC;
      const uint32_t idM = ptx::idesc_f16_f32(kTcTilePx, M);
      // Low descriptor words of the weight block of every (kx, chunk); the A operand of a
      // slot is its base word plus a compile-time offset (all shared addresses are below
      // 256 KB, so adding to the 14-bit start field never carries).
      uint32_t bv[3][Cfg::N];
#pragma unroll
      for (int kx = 0; kx < 3; ++kx)
#pragma unroll
        for (int k = 0; k < Cfg::N; ++k) bv[kx][k] = kx < NKX ? ptx::desc_lo(sW_u + a.wofs[kx * Cfg::N + k]) : 0u;
      bool ok = ptx::mbar_wait(ptx::smem_u32(wbar), 0, abort_flag, a.wait_limit_ns);
      SegIter it{pp == 0 ? t0 : tm, pp == 0 ? tm : t1, a.H};
      Segment sg;
      uint32_t obase = 0;
      RingPos fp;
      // Input row j of a segment feeds output rows j, j-1, j-2 through kernel rows
      // ky = 0, 1, 2. Output row o lives in chunk ring(o) = -o mod NCH of this pipe's TMEM
      // half, so those outputs occupy consecutive chunks and one MMA of N = 3M per
      // (kx, k-block) covers all three (split in two where the window wraps).
      while (ok && it.next(sg)) {
        const int n = sg.yb - sg.ya;
        for (int j = 0; j <= n + 1 && ok; ++j, fp.step(S)) {
          const uint32_t slot = fp.slot;
          ok = ptx::mbar_wait(ptx::smem_u32(&pfull[slot]), fp.phase, abort_flag, a.wait_limit_ns);
          const int ky_lo = max(0, j - (n - 1)), ky_hi = min(2, j);
          if (ok && ky_lo == 0) {  // output row j starts here: bias-initialise its chunk
            const uint32_t o = obase + j, c = (NCH - (o & (NCH - 1))) & (NCH - 1);
            ok = ptx::mbar_wait(ptx::smem_u32(&pacce[c]), ((o >> lgA) & 1u) ^ 1u, abort_flag, a.wait_limit_ns);
            ptx::tc_fence_after();
            if (ok) ptx::mma_f16_ss(tbase + c * M, ones_desc, biasb_desc, idM, 0);
          }
          if (!ok) break;
          const uint32_t ohi = obase + j - ky_lo;
          const uint32_t chi = (NCH - (ohi & (NCH - 1))) & (NCH - 1);
          const uint32_t span = ky_hi - ky_lo + 1;
          const uint32_t n1 = min(span, NCH - chi), n2 = span - n1;
          const uint32_t d1 = tbase + chi * M, d2 = tbase;
          const uint32_t i1 = ptx::idesc_f16_f32(kTcTilePx, n1 * M), i2 = ptx::idesc_f16_f32(kTcTilePx, n2 * M);
          const uint32_t sl = alo0 + slot * slot16;
          // One branch per row, none per MMA.
          if (n2 == 0) {
            vert_row_mmas<Cfg, false, NKX>(sl, bv, M, ky_lo, n1, d1, d2, i1, i2);
          } else {
            vert_row_mmas<Cfg, true, NKX>(sl, bv, M, ky_lo, n1, d1, d2, i1, i2);
          }
          ptx::mma_commit(ptx::smem_u32(&pempty[slot]));
          if (ky_hi == 2) {  // output row j-2 received its last kernel row
            const uint32_t o = obase + j - 2, c = (NCH - (o & (NCH - 1))) & (NCH - 1);
            ptx::mma_commit(ptx::smem_u32(&paccf[c]));
          }
        }
        obase += n;
      }
      // Drain every issued MMA before the tensor memory is released.
      ptx::mma_commit(ptx::smem_u32(&donebar[pp]));
      volatile int never_abort = 0;
      ptx::mbar_wait(ptx::smem_u32(&donebar[pp]), 0, &never_abort, a.wait_limit_ns);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (warps 4..11; 4..19 when WIDE) ----------------
    ptx::griddep_wait();  // residual operands and the output buffer belong to earlier layers
    const int e = warp - 4;
    const int pp = WIDE ? (e >> 3) : (e >> 2);    // pipe
    const int q = warp & 3;                       // tensor-memory lane quarter this warp may access
    // 32-channel groups of this warp (the DepthToSpace tails have M <= 16: one)
    constexpr int KG = (WIDE || EPI == 1 || EPI == 3) ? 1 : 2;
    const int gsel = WIDE ? ((e >> 2) & 1) : 0;   // its first group
    const int ngroups = (a.MT + 31) / 32;
    const int act = ACT >= 0 ? ACT : a.act;
    // (the same 32 KB of staging either way: 8 warps x 4 KB, or 16 x 2 KB)
    uint8_t* stage = sStage + e * (WIDE ? kStageTile : a.stage_per_warp);
    uint64_t* paccf = accf + pp * kMaxAcc;
    uint64_t* pacce = acce + pp * kMaxAcc;
    const uint32_t tbase = tmem_base + pp * half_cols;
    const ConvTcOut& o = a.out;
    uint32_t acc_cnt = 0;
    SegIter it{pp == 0 ? t0 : tm, pp == 0 ? tm : t1, a.H};
    Segment sg;
    bool ok = true;
    bool stores_pending = false;
    // First residual operand through the staging tiles (output form 0): lane 0 TMA-loads
    // the tile of the next row as soon as this row's store has read the staging, and the
    // math adds it in place. res_row: the row whose tile is in flight or landed.
    // Compiled into the no-activation NHWC variant only (the residual convs of these
    // models have no activation): the ReLU / SiLU variants keep their registers.
    const bool rt = EPI == 0 && ACT == kActNone && a.res_tma != 0;
    const __half* lop1 = rt ? nullptr : a.add1;  // operands loaded per lane
    uint32_t res_cnt = 0;
    int res_row = -1;
    bool res_inflight = false;
    auto issue_res = [&](int xw_, int yy) {  // lane 0
      uint32_t bytes = 0;
      for (int k = 0; k < KG && gsel + k < ngroups; ++k) bytes += min(32, a.MT - (gsel + k) * 32) * 64;
      ptx::mbar_arrive_expect_tx(ptx::smem_u32(&rbar[e]), bytes);
      for (int k = 0; k < KG && gsel + k < ngroups; ++k) {
        const int g = gsel + k;
        const CUtensorMap* map = min(32, a.MT - g * 32) == 32 ? &a.res_map32 : &a.res_map16;
        ptx::tma_load_3d(ptx::smem_u32(stage + k * kStageTile), map, ptx::smem_u32(&rbar[e]), m0 + g * 32, xw_, yy);
      }
    };
    while (ok && it.next(sg)) {
      // first pixel of this warp's 32 (EPI 3: sub-tile q, from one pixel left of its outputs)
      const int xw = EPI == 3 ? sg.strip * kStride - 1 + q * kKxnSubStep : sg.strip * kTcTilePx + q * 32;
      const int x = xw + lane;
      const bool valid = EPI == 3 ? (lane >= 1 && lane <= kKxnSubStep && x < a.W) : x < a.W;
      const bool wl = xw < a.W;  // this warp stores anything in this strip
      for (int y = sg.ya; y < sg.yb; ++y) {
        // accumulator of this output row: consecutive rows sit in descending chunks
        const uint32_t acc = (NACC - (acc_cnt & (NACC - 1))) & (NACC - 1);
        const size_t pix = static_cast<size_t>(y) * a.W + (valid ? x : 0);
        uint4 pre[2][2][4];  // [operand][channel group][8 channels]
        if constexpr (EPI == 0) {
          if (rt && wl && res_row != y) {  // first row of a segment: request its tile now
            if (lane == 0) {
              if (stores_pending) ptx::bulk_wait_group_read0();
              issue_res(xw, y);
            }
            __syncwarp();
            res_row = y;
            res_inflight = true;
          }
          if (valid && (lop1 || a.add2)) {
            // Residual lines of the row two ahead go to L2 now; this row's residual
            // operands are loaded into registers before the accumulator wait.
            if (y + 2 < sg.yb) {
#pragma unroll
              for (int k2 = 0; k2 < KG; ++k2) {
                const int g2 = gsel + k2;
                if (g2 >= ngroups) break;
                const size_t off = (pix + 2 * static_cast<size_t>(a.W)) * a.M + m0 + g2 * 32;
                if (lop1) ptx::prefetch_l2(lop1 + off);
                if (a.add2) ptx::prefetch_l2(a.add2 + off);
              }
            }
#pragma unroll
            for (int k2 = 0; k2 < KG; ++k2) {
              const int g2 = gsel + k2;
              if (g2 >= ngroups) break;
              const int cw = min(32, a.MT - g2 * 32);
              const size_t off = pix * a.M + m0 + g2 * 32;
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                if (i * 8 >= cw) break;
                if (lop1) pre[0][k2][i] = __ldg(reinterpret_cast<const uint4*>(lop1 + off + i * 8));
                if (a.add2) pre[1][k2][i] = __ldg(reinterpret_cast<const uint4*>(a.add2 + off + i * 8));
              }
            }
          }
        }
        int w_ok = 0;
        if (lane == 0)
          w_ok = ptx::mbar_wait(ptx::smem_u32(&paccf[acc]), (acc_cnt >> lgA) & 1u, abort_flag, a.wait_limit_ns) ? 1 : 0;
        w_ok = __shfl_sync(0xffffffffu, w_ok, 0);
        if (!w_ok) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        if constexpr (EPI == 0) {
          if (stores_pending) {
            if (lane == 0) ptx::bulk_wait_group_read0();  // the staging tiles are free again
            __syncwarp();
          }
        }
        // Every channel group of this warp's lane quarter (M <= 64: at most 2 groups) is read
        // out of TMEM first and the accumulator released at once: each pipe's ring has only
        // one chunk beyond the three-row window, so the MMA issuer waits on this release.
        uint32_t rrs[2][32];
#pragma unroll
        for (int k = 0; k < KG; ++k) {
          const int g = gsel + k;
          if (g >= ngroups) break;
          const uint32_t taddr = tbase + (static_cast<uint32_t>(q * 32) << 16) + acc * M + g * 32;
          if (min(32, a.MT - g * 32) < 32) {
            ptx::tmem_ld_32x32b_x16(taddr, rrs[k]);
          } else if (M & 31u) {  // 48-column chunks: 16-column loads at 16-aligned columns
            ptx::tmem_ld_32x32b_x16(taddr, rrs[k]);
            ptx::tmem_ld_32x32b_x16_hi(taddr + 16, rrs[k]);
          } else {
            ptx::tmem_ld_32x32b_x32(taddr, rrs[k]);
          }
        }
        ptx::tmem_wait_ld();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(&pacce[acc]));
        if (rt && wl) {  // this row's residual tile in the staging
          const bool r_ok = ptx::mbar_wait(ptx::smem_u32(&rbar[e]), res_cnt & 1u, abort_flag, a.wait_limit_ns);
          if (!__all_sync(0xffffffffu, r_ok)) {
            ok = false;
            break;
          }
          ++res_cnt;
          res_inflight = false;
        }
#pragma unroll
        for (int k = 0; k < KG; ++k) {
          const int g = gsel + k;
          if (g >= ngroups) break;
          const int cw = min(32, a.MT - g * 32);
          const uint32_t (&rr)[32] = rrs[k];
          const int cbase = g * 32;
          if constexpr (EPI == 0) {
            uint8_t* st = stage + k * kStageTile;
            const uint32_t rb = cw * 2;
#pragma unroll
            for (int j8 = 0; j8 < 32; j8 += 8) {
              if (j8 >= cw) break;
              uint32_t h[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                __half2 v = __floats2half2_rn(__uint_as_float(rr[j8 + 2 * i]), __uint_as_float(rr[j8 + 2 * i + 1]));
                h[i] = *reinterpret_cast<uint32_t*>(&v);
              }
              act8<ACT>(h);
              uint4* sp = reinterpret_cast<uint4*>(st + swz_granule(lane, j8 >> 3, rb));
              if (rt) {
                hadd8v(h, *sp);
                if (valid && a.add2) hadd8v(h, pre[1][k][j8 >> 3]);
              } else if (valid && a.add1) {
                hadd8v(h, pre[0][k][j8 >> 3]);
                if (a.add2) hadd8v(h, pre[1][k][j8 >> 3]);
              }
              *sp = make_uint4(h[0], h[1], h[2], h[3]);
            }
          } else if constexpr (EPI == 3) {
            // P_0 of the pixel on the left and P_2 of the pixel on the right (accumulator
            // columns kx * 4 + m), from the neighbouring lanes of this warp
            uint32_t ov[32];
#pragma unroll
            for (int m = 0; m < 4; ++m) {
              const float l = __shfl_up_sync(0xffffffffu, __uint_as_float(rr[m]), 1);
              const float r = __shfl_down_sync(0xffffffffu, __uint_as_float(rr[8 + m]), 1);
              ov[m] = __float_as_uint(l + __uint_as_float(rr[4 + m]) + r);
            }
            if (valid) store_dts2_nchw<1>(ov, act, o, y, x, a.H, a.W);
          } else if constexpr (EPI == 1) {
            if (valid) {
              switch (a.M >> 2) {
                case 1: store_dts2_nchw<1>(rr, act, o, y, x, a.H, a.W); break;
                case 2: store_dts2_nchw<2>(rr, act, o, y, x, a.H, a.W); break;
                case 3: store_dts2_nchw<3>(rr, act, o, y, x, a.H, a.W); break;
                default: store_dts2_nchw<4>(rr, act, o, y, x, a.H, a.W); break;
              }
            }
          } else {
            if (valid) {
              // General narrow outputs: per-element DepthToSpace (DCR) / clip / dtype / layout.
              const int b = o.dts_b;
              const int cout = a.M / (b * b);
              const long long Ho = static_cast<long long>(a.H) * b, Wo = static_cast<long long>(a.W) * b;
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const int m = m0 + cbase + j;
                if (j >= cw || m >= a.M) break;
                float t = act1(r16(__uint_as_float(rr[j])), act);
                if (a.add1) t = r16(t + __half2float(a.add1[pix * a.M + m]));
                if (a.add2) t = r16(t + __half2float(a.add2[pix * a.M + m]));
                if (o.clip) t = fminf(fmaxf(t, o.clip_lo), o.clip_hi);
                const int rq = m / cout, c = m - rq * cout;
                const int r_ = rq / b, q_ = rq - r_ * b;
                const long long oy = static_cast<long long>(y) * b + r_, ox = static_cast<long long>(x) * b + q_;
                const long long idx =
                    o.nchw ? ((static_cast<long long>(c) * Ho + oy) * Wo + ox) : ((oy * Wo + ox) * cout + c);
                if (o.fp32) static_cast<float*>(o.ptr)[idx] = t;
                else static_cast<__half*>(o.ptr)[idx] = __float2half_rn(t);
              }
            }
          }
        }
        if constexpr (EPI == 0) {
          ptx::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && xw < a.W) {
            for (int k = 0; k < KG && gsel + k < ngroups; ++k) {
              const int g = gsel + k;
              const int cw = min(32, a.MT - g * 32);
              const uint32_t src = ptx::smem_u32(stage + k * kStageTile);
              const CUtensorMap* map = cw == 32 ? &a.out_map32 : &a.out_map16;
              if (a.reduce_out) ptx::tma_reduce_add_3d(map, src, m0 + g * 32, xw, y);
              else ptx::tma_store_3d(map, src, m0 + g * 32, xw, y);
            }
            ptx::bulk_commit_group();
          }
          stores_pending = true;
          if (rt && wl && y + 1 < sg.yb) {  // next row's tile, once this store has read the staging
            if (lane == 0) {
              ptx::bulk_wait_group_read0();
              issue_res(xw, y + 1);
            }
            __syncwarp();
            res_row = y + 1;
            res_inflight = true;
          }
        }
        ++acc_cnt;
      }
    }
    if constexpr (EPI == 0) {
      if (res_inflight) {  // only after an abort: let the requested tile land before exit
        volatile int never_abort = 0;
        ptx::mbar_wait(ptx::smem_u32(&rbar[e]), res_cnt & 1u, &never_abort, a.wait_limit_ns);
      }
      if (lane == 0) ptx::bulk_wait_group0();
    }
    __syncwarp();
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, a.tmem_cols);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicOr(a.status, 1u);
}

// All output variants of one chunk geometry: the standard formulation (conv3x3_tc_kernel)
// and the vertical window (conv3x3_tc_vert2_kernel).
template <int NC64, int NC32, int NC16>
KernelFn pick(bool vert, int variant) {
  if (vert) {
    switch (variant) {
      case 0: return conv3x3_tc_vert2_kernel<NC64, NC32, NC16, 0, kActNone, 0>;
      case 1: return conv3x3_tc_vert2_kernel<NC64, NC32, NC16, 0, kActRelu, 0>;
      case 2: return conv3x3_tc_vert2_kernel<NC64, NC32, NC16, 0, kActSilu, 0>;
      case 3: return conv3x3_tc_vert2_kernel<NC64, NC32, NC16, 1, -1, 0>;
      case 4: return conv3x3_tc_vert2_kernel<NC64, NC32, NC16, 2, -1, 0>;
      case 6: return conv3x3_tc_vert2_kernel<NC64, NC32, NC16, 3, -1, 0>;
      default: return conv3x3_tc_vert2_kernel<NC64, NC32, NC16, 0, kActSilu, 1>;
    }
  }
  switch (variant) {
    case 0: return conv3x3_tc_kernel<NC64, NC32, NC16, 0, kActNone>;
    case 1: return conv3x3_tc_kernel<NC64, NC32, NC16, 0, kActRelu>;
    case 2: return conv3x3_tc_kernel<NC64, NC32, NC16, 0, kActSilu>;
    case 3: return conv3x3_tc_kernel<NC64, NC32, NC16, 1, -1>;
    default: return conv3x3_tc_kernel<NC64, NC32, NC16, 2, -1>;
  }
}

}  // namespace tck
}  // namespace ah
