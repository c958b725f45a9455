// Two-SM (cta_group::2) vertical-window 3x3 convolution for 64 -> 64 channel layers with
// NHWC output: the block convs that dominate an R8F64 frame.
//
// Same formulation as conv3x3_tc_vert2_kernel (conv_tc_kernel.cuh): every input row is read
// once, and one MMA per (kx, k-block) multiplies it against the three kernel rows ky stacked
// along N, into three consecutive accumulator chunks of a TMEM ring. What changes is the MMA
// shape. The single-SM kernel is bound by the shared-memory operand traffic of its
// 128 x 192 x 16 MMAs: the weights (B) are re-read by every MMA, and they are half of
// those reads. Here a cluster of two CTAs on two SMs issues 256 x N x 16 MMAs:
//  * each CTA stages its own 128-pixel half of a 256-pixel row segment (A rows 0-127 from the
//    even CTA's shared memory, 128-255 from the odd one's);
//  * each CTA holds half of every weight block, N/2 columns at the same shared-memory offset;
//  * each CTA's TMEM holds its 128 pixel rows of the accumulators.
// Per SM, the weight bytes read per FLOP halve. The even CTA's thread issues the MMAs for both.
//
// Weight layout: an MMA over the kernel rows [a, a + n) of the stacked [ky0; ky1; ky2]
// block (N = 64 n) reads, in CTA r, the stacked rows [64a + 32nr, 64a + 32n(r + 1)), so each
// CTA keeps one block per contiguous ky range ("piece"): (a, n) = (0,1), (0,2), (0,3),
// (1,1), (1,2), (2,1). That is 320 rows of 128 B per kx, 120 KB.
//
// Synchronisation across the pair:
//  * input rows: both CTAs' TMA loads complete on the even CTA's full barrier
//    (cp.async.bulk.tensor .cta_group::2), which the even producer arms for both;
//  * MMA completion (slot free, accumulator full): tcgen05.commit .multicast::cluster to the
//    same barrier in both CTAs;
//  * accumulator released: the epilogue warps of both CTAs arrive on the even CTA's barrier
//    (count 8);
//  * weights: the odd CTA tells the even issuer once its half has landed.
// Cluster barriers bracket the kernel: after the barrier initialisation, and before TMEM is
// freed and the CTAs exit (no CTA leaves while its peer's MMAs may read its shared memory).
// Every mbarrier wait is time-bounded, as in the single-SM kernels.

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "kernels.h"
#include "ptx.cuh"

namespace ah {

namespace {

// Warps: 0 / 3 = TMA producers of pipe 0 / 1 (both CTAs); 1 / 2 = MMA issuers of pipe 0 / 1
// (even CTA; warp 1 of both CTAs allocates TMEM); 4-7 / 8-11 = epilogues of pipe 0 / 1.
// Two row pipelines per pair, as in the single-SM kernel: while one issuer waits on its
// synchronisation chain, the other's MMAs keep the tensor cores busy.
constexpr int kPThreads = 384;
constexpr int kPSlots = 2;          // input-row slots per pipe and CTA
constexpr int kPSlotBytes = 17408;  // 130 pixels x 128 B, 1024-aligned
constexpr int kPPieceRows = 320;    // weight rows per kx (all pieces)
constexpr int kPKxBytes = kPPieceRows * 128;
constexpr int kPNacc = 4;           // accumulator chunks of 64 columns per pipe (256 TMEM columns)
constexpr int kPOffW = 0;
constexpr int kPOffA = kPOffW + 3 * kPKxBytes;
constexpr int kPOffOnes = kPOffA + 2 * kPSlots * kPSlotBytes;
constexpr int kPOffBias = kPOffOnes + 4096;
constexpr int kPOffStage = kPOffBias + 1024;
constexpr int kPOffBars = kPOffStage + 8 * 2 * 2048;
constexpr int kPSmem = kPOffBars + 256 + 1024;

// Row offset of the piece (a, n) inside a kx block.
__host__ __device__ constexpr int piece_row(int a, int n) {
  return a == 0 ? (n == 1 ? 0 : (n == 2 ? 32 : 96)) : (a == 1 ? (n == 1 ? 192 : 224) : 288);
}

struct PairArgs {
  CUtensorMap in_map;     // input NHWC, box {64 ch, 130 px, 1 row}, 128B swizzle
  CUtensorMap out_map32;  // output NHWC, box {32 ch, 32 px, 1 row}, 64B swizzle
  const uint8_t* wpack;   // [2 ranks][3 kx][320 rows][128 B]
  const float* bias;      // 64
  const __half* add1;
  const __half* add2;
  uint32_t* status;
  int H, W, act, reduce_out;
  long long rows_total;   // (256-pixel strips) x H
  unsigned long long wait_limit_ns;
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Shared::cluster address of this CTA's shared variable `laddr` in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t laddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(laddr), "r"(rank));
  return r;
}

__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// TMA tile load whose completion bytes count on the even CTA's barrier (cta_group::2 form;
// `bar` is a shared::cluster address in the even CTA).
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1,
                                                 int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void mma_pair(uint32_t d, uint32_t a_lo, uint32_t a_hi, uint32_t b_lo, uint32_t b_hi,
                                         uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .b64 ad, bd;\n\t.reg .pred p;\n\t"
      "mov.b64 ad, {%1, %2};\n\t"
      "mov.b64 bd, {%3, %4};\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], ad, bd, %5, p;\n\t}" ::"r"(d),
      "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(acc)
      : "memory");
}

// Arrive once on the barrier at shared offset `bar` in both CTAs when this thread's prior
// tcgen05 operations (of the pair) complete.
__device__ __forceinline__ void commit_pair_both(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
          bar)
      : "memory");
}

__device__ __forceinline__ void commit_pair_local(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ uint32_t swz(uint32_t r, uint32_t j, uint32_t rb) {
  const uint32_t phase = rb == 128 ? (r & 7u) : (rb == 64 ? ((r >> 1) & 3u) : ((r >> 2) & 1u));
  return r * rb + ((j ^ phase) << 4);
}

__device__ __forceinline__ void hadd8(uint32_t (&h)[4], const uint4& u) {
  const uint32_t* q = reinterpret_cast<const uint32_t*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 v = __hadd2(*reinterpret_cast<__half2*>(&h[i]), *reinterpret_cast<const __half2*>(&q[i]));
    h[i] = *reinterpret_cast<uint32_t*>(&v);
  }
}

template <int ACT>
__device__ __forceinline__ void act8p(uint32_t (&h)[4]) {
  if constexpr (ACT == kActSilu) {
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

template <int ACT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPThreads, 1)
    conv3x3_pair_kernel(const __grid_constant__ PairArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sW = smem + kPOffW;
  uint8_t* sA = smem + kPOffA;  // pipe p, slot s at sA + (p * kPSlots + s) * kPSlotBytes
  uint8_t* sOnes = smem + kPOffOnes;
  uint8_t* sBias = smem + kPOffBias;
  uint8_t* sStage = smem + kPOffStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kPOffBars);
  uint64_t* full = bars;                     // [2][kPSlots], used in the even CTA
  uint64_t* empty = full + 2 * kPSlots;      // [2][kPSlots], both CTAs
  uint64_t* accf = empty + 2 * kPSlots;      // [2][kPNacc], both CTAs
  uint64_t* acce = accf + 2 * kPNacc;        // [2][kPNacc], used in the even CTA (count 8)
  uint64_t* wbar = acce + 2 * kPNacc;        // this CTA's weight half
  uint64_t* wpeer = wbar + 1;                // even CTA: the odd CTA's weights landed
  uint64_t* donebar = wpeer + 1;             // [2] even CTA: every MMA of a pipe drained
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(donebar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool lead = rank == 0;
  ptx::griddep_launch_dependents();

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2 * kPSlots; ++i) {
      ptx::mbar_init(ptx::smem_u32(&full[i]), 1);
      ptx::mbar_init(ptx::smem_u32(&empty[i]), 1);
    }
    for (int i = 0; i < 2 * kPNacc; ++i) {
      ptx::mbar_init(ptx::smem_u32(&accf[i]), 1);
      ptx::mbar_init(ptx::smem_u32(&acce[i]), 8);  // the pipe's 4 epilogue warps in each CTA
    }
    ptx::mbar_init(ptx::smem_u32(wbar), 1);
    ptx::mbar_init(ptx::smem_u32(wpeer), 1);
    ptx::mbar_init(ptx::smem_u32(&donebar[0]), 1);
    ptx::mbar_init(ptx::smem_u32(&donebar[1]), 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if ((warp == 0 || warp == 3) && lane == 0) ptx::prefetch_tensormap(&a.in_map);
  if (warp == 1) {  // the pair's TMEM: the same warp of both CTAs, the same slot offset
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(ptx::smem_u32(tmem_slot)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  // Bias operands: a ones column for this CTA's 128 pixel rows, and this CTA's half of the
  // bias (channels 32 rank .. + 31) as column 0 of the B rows.
  for (int r = threadIdx.x; r < 128; r += blockDim.x) {
    uint4* row = reinterpret_cast<uint4*>(sOnes + r * 32);
    row[0] = make_uint4(0, 0, 0, 0);
    row[1] = make_uint4(0, 0, 0, 0);
    *reinterpret_cast<__half*>(sOnes + swz(r, 0, 32)) = __float2half(1.f);
  }
  for (int r = threadIdx.x; r < 32; r += blockDim.x) {
    uint4* row = reinterpret_cast<uint4*>(sBias + r * 32);
    row[0] = make_uint4(0, 0, 0, 0);
    row[1] = make_uint4(0, 0, 0, 0);
    *reinterpret_cast<__half*>(sBias + swz(r, 0, 32)) = __float2half(a.bias[32 * rank + r]);
  }
  ptx::fence_proxy_async_smem();
  ptx::tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any cross-CTA arrive or load
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // The cluster's contiguous (256-pixel strip, row) range, split between the two pipes.
  const long long nclus = gridDim.x / 2;
  const long long cl = blockIdx.x / 2;
  const long long t0 = cl * a.rows_total / nclus;
  const long long t1 = (cl + 1) * a.rows_total / nclus;
  const long long tm = (t0 + t1) / 2;

  if (warp == 0 || warp == 3) {
    // ---------------- TMA producers (both CTAs) ----------------
    const int pp = warp == 0 ? 0 : 1;
    if (lane == 0) {
      bool ok = true;
      if (pp == 0) {
        ptx::mbar_arrive_expect_tx(ptx::smem_u32(wbar), 3 * kPKxBytes);
        for (int kx = 0; kx < 3; ++kx)
          ptx::bulk_load(ptx::smem_u32(sW + kx * kPKxBytes),
                         a.wpack + (static_cast<size_t>(rank) * 3 + kx) * kPKxBytes, kPKxBytes, ptx::smem_u32(wbar));
        if (!lead) {  // tell the even issuers this half of the weights is in place
          ok = ptx::mbar_wait(ptx::smem_u32(wbar), 0, abort_flag, a.wait_limit_ns);
          if (ok) mbar_arrive_remote(map_to_rank(ptx::smem_u32(wpeer), 0));
        }
      }
      ptx::griddep_wait();  // the input rows come from the previous layer
      uint64_t* pfull = full + pp * kPSlots;
      uint64_t* pempty = empty + pp * kPSlots;
      uint8_t* pA = sA + static_cast<size_t>(pp) * kPSlots * kPSlotBytes;
      const uint32_t full0 = map_to_rank(ptx::smem_u32(&pfull[0]), 0);
      uint32_t g = 0, slot = 0, phase = 0;
      for (long long t = pp == 0 ? t0 : tm, tend = pp == 0 ? tm : t1; t < tend && ok;) {
        const int strip = static_cast<int>(t / a.H), ya = static_cast<int>(t % a.H);
        const int yb = static_cast<int>(std::min<long long>(a.H, ya + (tend - t)));
        t = static_cast<long long>(strip) * a.H + yb;
        const int x0 = strip * 256 + 128 * static_cast<int>(rank) - 1;
        for (int r = ya - 1; r <= yb; ++r, ++g) {
          if (!ptx::mbar_wait(ptx::smem_u32(&pempty[slot]), phase ^ 1u, abort_flag, a.wait_limit_ns)) {
            ok = false;
            break;
          }
          if (lead) ptx::mbar_arrive_expect_tx(ptx::smem_u32(&pfull[slot]), 2 * 130 * 128);
          tma_load_3d_pair(ptx::smem_u32(pA + slot * kPSlotBytes), &a.in_map, full0 + slot * 8u, 0, x0, r);
          if (++slot == kPSlots) {
            slot = 0;
            phase ^= 1u;
          }
        }
      }
      // No TMA write in flight at exit: the even CTA waits (bounded) on the last loads of
      // both CTAs; the odd CTA's loads are covered by the cluster barrier after that wait.
      if (lead) {
        volatile int never_abort = 0;
        const uint32_t first = g > static_cast<uint32_t>(kPSlots) ? g - kPSlots : 0u;
        for (uint32_t j = first; j < g; ++j)
          ptx::mbar_wait(ptx::smem_u32(&pfull[j % kPSlots]), (j / kPSlots) & 1u, &never_abort, a.wait_limit_ns);
      }
    }
  } else if (warp == 1 || warp == 2) {
    // ---------------- MMA issuers (even CTA) ----------------
    const int pp = warp - 1;
    if (lane == 0 && lead) {
      uint64_t* pfull = full + pp * kPSlots;
      uint64_t* pempty = empty + pp * kPSlots;
      uint64_t* paccf = accf + pp * kPNacc;
      uint64_t* pacce = acce + pp * kPNacc;
      const uint32_t tbase = tmem_base + pp * 256;
      const uint32_t sA_u = ptx::smem_u32(sA + static_cast<size_t>(pp) * kPSlots * kPSlotBytes);
      const uint32_t sW_u = ptx::smem_u32(sW);
      const uint32_t ones_lo = ptx::desc_lo(ptx::smem_u32(sOnes)), bias_lo = ptx::desc_lo(ptx::smem_u32(sBias));
      const uint32_t hi32 = ptx::desc_hi(256, 6), hi128 = ptx::desc_hi(1024, 2);
      const uint32_t alo0 = ptx::desc_lo(sA_u);
      const uint32_t wlo0 = ptx::desc_lo(sW_u);
      constexpr uint32_t NCH = kPNacc;
      const uint32_t id_bias = ptx::idesc_f16_f32(256, 64);
      bool ok = ptx::mbar_wait(ptx::smem_u32(wbar), 0, abort_flag, a.wait_limit_ns);
      if (ok) ok = ptx::mbar_wait(ptx::smem_u32(wpeer), 0, abort_flag, a.wait_limit_ns);
      uint32_t obase = 0, slot = 0, phase = 0;
      for (long long t = pp == 0 ? t0 : tm, tend = pp == 0 ? tm : t1; t < tend && ok;) {
        const int strip = static_cast<int>(t / a.H), ya = static_cast<int>(t % a.H);
        const int yb = static_cast<int>(std::min<long long>(a.H, ya + (tend - t)));
        t = static_cast<long long>(strip) * a.H + yb;
        const int n = yb - ya;
        for (int j = 0; j <= n + 1 && ok; ++j) {
          ok = ptx::mbar_wait(ptx::smem_u32(&pfull[slot]), phase, abort_flag, a.wait_limit_ns);
          const int ky_lo = max(0, j - (n - 1)), ky_hi = min(2, j);
          if (ok && ky_lo == 0) {  // output row j starts here: bias-initialise its chunk
            const uint32_t o = obase + j, c = (NCH - (o & (NCH - 1))) & (NCH - 1);
            ok = ptx::mbar_wait(ptx::smem_u32(&pacce[c]), ((o >> 2) & 1u) ^ 1u, abort_flag, a.wait_limit_ns);
            ptx::tc_fence_after();
            if (ok) mma_pair(tbase + c * 64, ones_lo, hi32, bias_lo, hi32, id_bias, 0);
          }
          if (!ok) break;
          const uint32_t ohi = obase + j - ky_lo;
          const uint32_t chi = (NCH - (ohi & (NCH - 1))) & (NCH - 1);
          const uint32_t span = ky_hi - ky_lo + 1;
          const uint32_t n1 = min(span, NCH - chi), n2 = span - n1;
          const uint32_t d1 = tbase + chi * 64, d2 = tbase;
          const uint32_t i1 = ptx::idesc_f16_f32(256, n1 * 64), i2 = ptx::idesc_f16_f32(256, (n2 ? n2 : 1) * 64);
          const uint32_t p1 = static_cast<uint32_t>(piece_row(ky_lo, n1)) * 8u;  // rows x 128 B in 16-B units
          const uint32_t p2 = n2 ? static_cast<uint32_t>(piece_row(ky_lo + n1, n2)) * 8u : 0u;
          const uint32_t sl = alo0 + slot * (kPSlotBytes >> 4);
          if (n2 == 0) {  // one branch per row, none per MMA
#pragma unroll
            for (int kx = 0; kx < 3; ++kx)
#pragma unroll
              for (int kb = 0; kb < 4; ++kb)
                mma_pair(d1, sl + ((kx * 128 + kb * 32) >> 4), hi128, wlo0 + ((kx * kPKxBytes + kb * 32) >> 4) + p1,
                         hi128, i1, 1);
          } else {
#pragma unroll
            for (int kx = 0; kx < 3; ++kx)
#pragma unroll
              for (int kb = 0; kb < 4; ++kb) {
                const uint32_t alo = sl + ((kx * 128 + kb * 32) >> 4);
                const uint32_t wb = wlo0 + ((kx * kPKxBytes + kb * 32) >> 4);
                mma_pair(d1, alo, hi128, wb + p1, hi128, i1, 1);
                mma_pair(d2, alo, hi128, wb + p2, hi128, i2, 1);
              }
          }
          commit_pair_both(ptx::smem_u32(&pempty[slot]));
          if (ky_hi == 2) {  // output row j-2 received its last kernel row
            const uint32_t o = obase + j - 2, c = (NCH - (o & (NCH - 1))) & (NCH - 1);
            commit_pair_both(ptx::smem_u32(&paccf[c]));
          }
          if (++slot == kPSlots) {
            slot = 0;
            phase ^= 1u;
          }
        }
        obase += n;
      }
      commit_pair_local(ptx::smem_u32(&donebar[pp]));
      volatile int never_abort = 0;
      ptx::mbar_wait(ptx::smem_u32(&donebar[pp]), 0, &never_abort, a.wait_limit_ns);
    }
    __syncwarp();
  } else {
    // ---------------- epilogues (warps 4-7: pipe 0, 8-11: pipe 1; both CTAs) ----------------
    ptx::griddep_wait();  // residual operands and the output buffer belong to earlier layers
    const int e = warp - 4;
    const int pp = e >> 2;
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    uint8_t* stage = sStage + e * 2 * 2048;
    const uint32_t tbase = tmem_base + pp * 256;
    uint64_t* paccf = accf + pp * kPNacc;
    const uint32_t acce0 = map_to_rank(ptx::smem_u32(&acce[pp * kPNacc]), 0);
    uint32_t acc_cnt = 0;
    bool ok = true;
    bool stores_pending = false;
    for (long long t = pp == 0 ? t0 : tm, tend = pp == 0 ? tm : t1; t < tend && ok;) {
      const int strip = static_cast<int>(t / a.H), ya = static_cast<int>(t % a.H);
      const int yb = static_cast<int>(std::min<long long>(a.H, ya + (tend - t)));
      t = static_cast<long long>(strip) * a.H + yb;
      const int xw = strip * 256 + 128 * static_cast<int>(rank) + q * 32;
      const int x = xw + lane;
      const bool valid = x < a.W;
      for (int y = ya; y < yb; ++y) {
        const uint32_t acc = (kPNacc - (acc_cnt & (kPNacc - 1))) & (kPNacc - 1);
        const size_t pix = static_cast<size_t>(y) * a.W + (valid ? x : 0);
        uint4 pre[2][2][4];
        if (valid && a.add1) {
          if (y + 2 < yb) {
#pragma unroll
            for (int g = 0; g < 2; ++g) {
              const size_t off = (pix + 2 * static_cast<size_t>(a.W)) * 64 + g * 32;
              ptx::prefetch_l2(a.add1 + off);
              if (a.add2) ptx::prefetch_l2(a.add2 + off);
            }
          }
#pragma unroll
          for (int g = 0; g < 2; ++g)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const size_t off = pix * 64 + g * 32 + i * 8;
              pre[0][g][i] = __ldg(reinterpret_cast<const uint4*>(a.add1 + off));
              if (a.add2) pre[1][g][i] = __ldg(reinterpret_cast<const uint4*>(a.add2 + off));
            }
        }
        int w_ok = 0;
        if (lane == 0)
          w_ok = ptx::mbar_wait(ptx::smem_u32(&paccf[acc]), (acc_cnt >> 2) & 1u, abort_flag, a.wait_limit_ns) ? 1 : 0;
        w_ok = __shfl_sync(0xffffffffu, w_ok, 0);
        if (!w_ok) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        if (stores_pending) {
          if (lane == 0) ptx::bulk_wait_group_read0();  // the staging tiles are free again
          __syncwarp();
        }
        uint32_t rrs[2][32];
#pragma unroll
        for (int g = 0; g < 2; ++g)
          ptx::tmem_ld_32x32b_x32(tbase + (static_cast<uint32_t>(q * 32) << 16) + acc * 64 + g * 32, rrs[g]);
        ptx::tmem_wait_ld();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(acce0 + acc * 8u);  // the even CTA's barrier
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          uint8_t* st = stage + g * 2048;
#pragma unroll
          for (int j8 = 0; j8 < 32; j8 += 8) {
            uint32_t h[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              __half2 v = __floats2half2_rn(__uint_as_float(rrs[g][j8 + 2 * i]), __uint_as_float(rrs[g][j8 + 2 * i + 1]));
              h[i] = *reinterpret_cast<uint32_t*>(&v);
            }
            act8p<ACT>(h);
            if (valid && a.add1) {
              hadd8(h, pre[0][g][j8 >> 3]);
              if (a.add2) hadd8(h, pre[1][g][j8 >> 3]);
            }
            *reinterpret_cast<uint4*>(st + swz(lane, j8 >> 3, 64)) = make_uint4(h[0], h[1], h[2], h[3]);
          }
        }
        ptx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && xw < a.W) {
          for (int g = 0; g < 2; ++g) {
            const uint32_t src = ptx::smem_u32(stage + g * 2048);
            if (a.reduce_out) ptx::tma_reduce_add_3d(&a.out_map32, src, g * 32, xw, y);
            else ptx::tma_store_3d(&a.out_map32, src, g * 32, xw, y);
          }
          ptx::bulk_commit_group();
        }
        stores_pending = true;
        ++acc_cnt;
      }
    }
    if (lane == 0) ptx::bulk_wait_group0();
    __syncwarp();
  }

  ptx::tc_fence_before();
  __syncthreads();
  cluster_sync();  // the pair's MMAs, loads and remote arrivals are all done
  if (warp == 1) {
    ptx::tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(512) : "memory");
  }
  if (threadIdx.x == 0 && *abort_flag) atomicOr(a.status, 1u);
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn pair_encode_fn() {
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

bool encode_nhwc(EncodeTiledFn enc, CUtensorMap* map, const void* base, int W, int H, int box_c, int box_px,
                 CUtensorMapSwizzle sw, std::string* err) {
  cuuint64_t gdim[3] = {64, static_cast<cuuint64_t>(W), static_cast<cuuint64_t>(H)};
  cuuint64_t gstride[2] = {64 * 2, static_cast<cuuint64_t>(W) * 64 * 2};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box_c), static_cast<cuuint32_t>(box_px), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), gdim, gstride, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    if (err) *err = "cuTensorMapEncodeTiled failed (code " + std::to_string(static_cast<int>(r)) + ")";
    return false;
  }
  return true;
}

uint32_t swz_host(uint32_t r, uint32_t j) { return r * 128u + ((j ^ (r & 7u)) << 4); }

}  // namespace

bool pair_supported(int C, int M) { return C == 64 && M == 64; }

cudaError_t pair_upload(const uint16_t* w_oihw, const float* bias, int C, int M, PairWeights* out) {
  if (!pair_supported(C, M)) return cudaErrorInvalidValue;
  // [rank][kx][piece rows][128 B]: piece (a, n) of rank r holds the stacked rows
  // [64a + 32nr, 64a + 32n(r + 1)) of the [ky0; ky1; ky2] block, stacked row = ky * 64 + m.
  std::vector<uint8_t> img(static_cast<size_t>(2) * 3 * kPKxBytes, 0);
  const int pa[6] = {0, 0, 0, 1, 1, 2}, pn[6] = {1, 2, 3, 1, 2, 1};
  for (int rk = 0; rk < 2; ++rk)
    for (int kx = 0; kx < 3; ++kx)
      for (int pi = 0; pi < 6; ++pi) {
        const int a0 = pa[pi], n = pn[pi];
        uint8_t* blk = img.data() + (static_cast<size_t>(rk) * 3 + kx) * kPKxBytes + piece_row(a0, n) * 128;
        for (int rl = 0; rl < 32 * n; ++rl) {
          const int srow = 64 * a0 + 32 * n * rk + rl;
          const int ky = srow / 64, m = srow % 64;
          for (int c = 0; c < 64; ++c) {
            const uint16_t v = w_oihw[(static_cast<size_t>(m) * C + c) * 9 + ky * 3 + kx];
            std::memcpy(blk + swz_host(rl, c / 8) + (c % 8) * 2, &v, 2);
          }
        }
      }
  cudaError_t e = cudaMalloc(&out->wpack, img.size());
  if (e != cudaSuccess) return e;
  e = cudaMemcpy(out->wpack, img.data(), img.size(), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return e;
  std::vector<float> b(64, 0.f);
  if (bias) std::memcpy(b.data(), bias, sizeof(float) * 64);
  e = cudaMalloc(&out->bias, sizeof(float) * 64);
  if (e != cudaSuccess) return e;
  return cudaMemcpy(out->bias, b.data(), sizeof(float) * 64, cudaMemcpyHostToDevice);
}

void pair_free(PairWeights* w) {
  if (w->wpack) cudaFree(w->wpack);
  if (w->bias) cudaFree(w->bias);
  w->wpack = nullptr;
  w->bias = nullptr;
}

bool pair_plan(const PairWeights* w, const __half* in, int H, int W, __half* out, int num_sms, PairPlan* P,
               std::string* err) {
  EncodeTiledFn enc = pair_encode_fn();
  if (!enc) {
    if (err) *err = "cuTensorMapEncodeTiled is unavailable from the CUDA driver";
    return false;
  }
  if ((reinterpret_cast<uintptr_t>(in) & 15u) || (reinterpret_cast<uintptr_t>(out) & 15u)) {
    if (err) *err = "two-SM conv buffers must be 16-byte aligned";
    return false;
  }
  if (!encode_nhwc(enc, &P->in_map, in, W, H, 64, 130, CU_TENSOR_MAP_SWIZZLE_128B, err)) return false;
  if (!encode_nhwc(enc, &P->out_map32, out, W, H, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B, err)) return false;
  P->w = w;
  P->H = H;
  P->W = W;
  P->out = out;
  P->rows_total = static_cast<long long>((W + 255) / 256) * H;
  long long nclus = std::max(1, num_sms / 2);
  if (nclus > P->rows_total) nclus = P->rows_total;
  P->grid_x = static_cast<int>(2 * nclus);
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    for (auto fn : {conv3x3_pair_kernel<kActNone>, conv3x3_pair_kernel<kActRelu>, conv3x3_pair_kernel<kActSilu>}) {
      const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kPSmem);
      if (e != cudaSuccess) attr_err = e;
    }
  });
  if (attr_err != cudaSuccess) {
    if (err) *err = std::string("cudaFuncSetAttribute failed: ") + cudaGetErrorString(attr_err);
    return false;
  }
  return true;
}

cudaError_t pair_launch(const PairPlan& P, const __half* add1, const __half* add2, int act, uint32_t* status,
                        cudaStream_t stream) {
  PairArgs a;
  std::memset(&a, 0, sizeof(a));
  a.in_map = P.in_map;
  a.out_map32 = P.out_map32;
  a.wpack = static_cast<const uint8_t*>(P.w->wpack);
  a.bias = P.w->bias;
  a.add1 = add1 ? add1 : add2;
  a.add2 = add1 ? add2 : nullptr;
  // In place: the output buffer is the last residual operand; its addition goes to
  // reduce-add stores instead of a load (fp16(r + t) == fp16(t + r)).
  const __half* last = a.add2 ? a.add2 : a.add1;
  if (last && static_cast<const void*>(last) == static_cast<const void*>(P.out)) {
    a.reduce_out = 1;
    if (a.add2) a.add2 = nullptr;
    else a.add1 = nullptr;
  }
  a.status = status;
  a.H = P.H;
  a.W = P.W;
  a.act = act;
  a.rows_total = P.rows_total;
  a.wait_limit_ns = 4000000000ull;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(P.grid_x);
  cfg.blockDim = dim3(kPThreads);
  cfg.dynamicSmemBytes = kPSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (act == kActRelu) return cudaLaunchKernelEx(&cfg, conv3x3_pair_kernel<kActRelu>, a);
  if (act == kActSilu) return cudaLaunchKernelEx(&cfg, conv3x3_pair_kernel<kActSilu>, a);
  return cudaLaunchKernelEx(&cfg, conv3x3_pair_kernel<kActNone>, a);
}

}  // namespace ah
