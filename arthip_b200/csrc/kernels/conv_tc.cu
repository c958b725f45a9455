// tcgen05 implicit-GEMM 3x3 convolution (stride 1, SAME padding) for sm_100a.
//
// Replaces the reference's gfx1100 Winograd WMMA kernel (src/common/hip_kernels.h:143-396)
// for every conv whose channel counts fit the tensor-core tiling (C and M multiples of 16).
//
// GEMM view: one output row segment of 128 pixels is the MMA M dimension, the output
// channels are N, and K = 9 taps x C input channels. Per output row the kernel issues
// 9 * C/16 tcgen05.mma (128 x MT x 16, fp16 in, fp32 accumulate in tensor memory).
//
// Data movement:
//  * input: one TMA tiled load per (input row, channel chunk) brings 130 pixels
//    (the 128-pixel tile plus a 1-pixel halo each side; out-of-range pixels and rows are
//    zero-filled by the TMA unit, which is exactly the conv's zero padding) into a ring of
//    row slots. Each staged row feeds three consecutive output rows (ky = 0,1,2); the
//    three horizontal taps (kx) read the same slot with the descriptor start moved by one
//    pixel row, so nothing is re-staged.
//  * weights: resident in shared memory for the whole (persistent) kernel, in the
//    swizzled K-major layout the MMA reads; packed once on the host.
//  * accumulators: a ring of NACC tensor-memory accumulators; the epilogue warps drain
//    one while the MMA warp fills the next.
//  * epilogue: tcgen05.ld -> +bias -> fp16 rounding (the conv node's output) -> ReLU or
//    SiLU -> up to two residual adds (each rounded to fp16, as the ONNX Add nodes are)
//    -> 16-byte NHWC stores.
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM allocator + MMA issuer
// (one thread), warps 2..5 = epilogue (each owns the TMEM lane quarter warp%4).
// Work: the (strip, row) space is split into contiguous ranges, one per CTA.

#include <algorithm>
#include <cstdio>
#include <cstring>

#include "kernels.h"
#include "ptx.cuh"

namespace ah {

namespace {

constexpr int kMaxSlots = 8;
constexpr int kMaxAcc = 4;
constexpr int kThreads = 192;
constexpr int kSmemLimit = 232448;  // 227 KB opt-in dynamic shared memory per block

struct ConvTcArgs {
  CUtensorMap maps[kTcMaxChunks];
  const uint8_t* wpack;
  const float* bias;
  const __half* add1;
  const __half* add2;
  __half* out;
  uint32_t* status;
  long long gofs[9 * kTcMaxChunks];
  int wofs[9 * kTcMaxChunks];
  int H, W, M, MT;
  int nchunks;
  int rowbytes[kTcMaxChunks];
  int layout[kTcMaxChunks];
  int kblocks[kTcMaxChunks];
  int c0[kTcMaxChunks];
  int slot_off[kTcMaxChunks];
  int slot_bytes;
  int slot_tx;  // bytes one row load delivers (all chunks, full boxes)
  int nslots;
  int w_smem_bytes;
  int n_strips;
  long long rows_total;
  int act;
  int desc_base_mode;
  int nacc, acc_stride;
  uint32_t tmem_cols;
};

struct Segment {
  int strip, ya, yb;
};

// Iterates the CTA's contiguous range of (strip, row) tiles as per-strip segments.
struct SegIter {
  long long t, t1;
  int H;
  __device__ bool next(Segment& s) {
    if (t >= t1) return false;
    s.strip = static_cast<int>(t / H);
    s.ya = static_cast<int>(t % H);
    const long long left = t1 - t;
    s.yb = static_cast<int>(min(static_cast<long long>(H), s.ya + left));
    t = static_cast<long long>(s.strip) * H + s.yb;
    return true;
  }
};

__device__ __forceinline__ float h2f(__half h) { return __half2float(h); }
__device__ __forceinline__ float r16(float v) { return __half2float(__float2half_rn(v)); }

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __half22float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
  return u;
}

__global__ void __launch_bounds__(kThreads, 1) conv3x3_tc_kernel(const __grid_constant__ ConvTcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sW = smem;
  uint8_t* sA = smem + a.w_smem_bytes;
  float* sBias = reinterpret_cast<float*>(sA + a.nslots * a.slot_bytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sBias + 256);
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
  const int S = a.nslots;
  const int NACC = a.nacc;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(ptx::smem_u32(&full[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&empty[s]), 1);
    }
    for (int i = 0; i < NACC; ++i) {
      ptx::mbar_init(ptx::smem_u32(&accf[i]), 1);
      ptx::mbar_init(ptx::smem_u32(&acce[i]), 4);
    }
    ptx::mbar_init(ptx::smem_u32(wbar), 1);
    ptx::mbar_init(ptx::smem_u32(donebar), 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    for (int k = 0; k < a.nchunks; ++k) ptx::prefetch_tensormap(&a.maps[k]);
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_u32(tmem_slot), a.tmem_cols);
    ptx::tmem_relinquish();
  }
  for (int i = threadIdx.x; i < a.MT; i += blockDim.x) sBias[i] = a.bias[m0 + i];
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const long long t0 = static_cast<long long>(blockIdx.x) * a.rows_total / gridDim.x;
  const long long t1 = static_cast<long long>(blockIdx.x + 1) * a.rows_total / gridDim.x;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      uint32_t wbytes = 0;
      for (int t = 0; t < 9; ++t)
        for (int k = 0; k < a.nchunks; ++k) wbytes += a.MT * a.rowbytes[k];
      ptx::mbar_arrive_expect_tx(ptx::smem_u32(wbar), wbytes);
      for (int t = 0; t < 9; ++t) {
        for (int k = 0; k < a.nchunks; ++k) {
          const int idx = t * a.nchunks + k;
          const uint8_t* src = a.wpack + a.gofs[idx] + static_cast<long long>(m0) * a.rowbytes[k];
          ptx::bulk_load(ptx::smem_u32(sW + a.wofs[idx]), src, a.MT * a.rowbytes[k], ptx::smem_u32(wbar));
        }
      }
      uint32_t g = 0;
      SegIter it{t0, t1, a.H};
      Segment sg;
      bool ok = true;
      while (ok && it.next(sg)) {
        const int x0 = sg.strip * kTcTilePx - 1;
        for (int r = sg.ya - 1; r <= sg.yb; ++r, ++g) {
          const uint32_t slot = g % S;
          if (!ptx::mbar_wait(ptx::smem_u32(&empty[slot]), ((g / S) & 1u) ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t fb = ptx::smem_u32(&full[slot]);
          ptx::mbar_arrive_expect_tx(fb, a.slot_tx);
          const uint32_t dst = ptx::smem_u32(sA + slot * a.slot_bytes);
          for (int k = 0; k < a.nchunks; ++k)
            ptx::tma_load_3d(dst + a.slot_off[k], &a.maps[k], fb, a.c0[k], x0, r);
        }
      }
      // Never leave a TMA write in flight at exit: wait (time-bounded) for the last loads.
      volatile int never_abort = 0;
      const uint32_t first = g > static_cast<uint32_t>(S) ? g - S : 0u;
      for (uint32_t j = first; j < g; ++j)
        ptx::mbar_wait(ptx::smem_u32(&full[j % S]), (j / S) & 1u, &never_abort);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = ptx::idesc_f16_f32(kTcTilePx, a.MT);
      const uint32_t sA_u = ptx::smem_u32(sA);
      const uint32_t sW_u = ptx::smem_u32(sW);
      bool ok = ptx::mbar_wait(ptx::smem_u32(wbar), 0, abort_flag);
      uint32_t g_base = 0, acc_cnt = 0;
      SegIter it{t0, t1, a.H};
      Segment sg;
      while (ok && it.next(sg)) {
        const int n = sg.yb - sg.ya;
        for (int i = 0; i < n && ok; ++i) {
          for (int ky = 0; ky < 3 && ok; ++ky) {
            const uint32_t gl = g_base + i + ky;
            ok = ptx::mbar_wait(ptx::smem_u32(&full[gl % S]), (gl / S) & 1u, abort_flag);
          }
          const uint32_t acc = acc_cnt % NACC;
          if (ok) ok = ptx::mbar_wait(ptx::smem_u32(&acce[acc]), ((acc_cnt / NACC) & 1u) ^ 1u, abort_flag);
          if (!ok) break;
          ptx::tc_fence_after();
          const uint32_t d = tmem_base + acc * a.acc_stride;
          uint32_t accumulate = 0;
          for (int ky = 0; ky < 3; ++ky) {
            const uint32_t a_slot = sA_u + ((g_base + i + ky) % S) * a.slot_bytes;
            for (int k = 0; k < a.nchunks; ++k) {
              const uint32_t rb = a.rowbytes[k];
              const uint32_t lay = a.layout[k];
              const uint32_t sbo = 8u * rb;
              const uint32_t a_chunk = a_slot + a.slot_off[k];
              for (int kx = 0; kx < 3; ++kx) {
                const uint32_t b_blk = sW_u + a.wofs[(ky * 3 + kx) * a.nchunks + k];
                for (int kb = 0; kb < a.kblocks[k]; ++kb) {
                  const uint64_t ad = ptx::smem_desc(a_chunk + kx * rb + kb * 32u, lay, sbo, a.desc_base_mode);
                  const uint64_t bd = ptx::smem_desc(b_blk + kb * 32u, lay, sbo, a.desc_base_mode);
                  ptx::mma_f16_ss(d, ad, bd, idesc, accumulate);
                  accumulate = 1;
                }
              }
            }
          }
          ptx::mma_commit(ptx::smem_u32(&accf[acc]));
          ptx::mma_commit(ptx::smem_u32(&empty[(g_base + i) % S]));
          ++acc_cnt;
        }
        if (!ok) break;
        ptx::mma_commit(ptx::smem_u32(&empty[(g_base + n) % S]));
        ptx::mma_commit(ptx::smem_u32(&empty[(g_base + n + 1) % S]));
        g_base += n + 2;
      }
      // Drain every issued MMA before the tensor memory is released.
      ptx::mma_commit(ptx::smem_u32(donebar));
      volatile int never_abort = 0;
      ptx::mbar_wait(ptx::smem_u32(donebar), 0, &never_abort);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int q = warp & 3;  // tensor-memory lane quarter this warp may access
    const int p = q * 32 + lane;
    uint32_t acc_cnt = 0;
    SegIter it{t0, t1, a.H};
    Segment sg;
    bool ok = true;
    while (ok && it.next(sg)) {
      const int x = sg.strip * kTcTilePx + p;
      const bool valid = x < a.W;
      for (int y = sg.ya; y < sg.yb; ++y) {
        const uint32_t acc = acc_cnt % NACC;
        int w_ok = 0;
        if (lane == 0) w_ok = ptx::mbar_wait(ptx::smem_u32(&accf[acc]), (acc_cnt / NACC) & 1u, abort_flag) ? 1 : 0;
        w_ok = __shfl_sync(0xffffffffu, w_ok, 0);
        if (!w_ok) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const size_t pix = static_cast<size_t>(y) * a.W + (valid ? x : 0);
        const size_t obase = pix * a.M + m0;
        for (int cc = 0; cc < a.MT; cc += 32) {
          uint32_t r[32];
          const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * a.acc_stride + cc;
          const int ncols = min(32, a.MT - cc);
          if (ncols == 32) ptx::tmem_ld_32x32b_x32(taddr, r);
          else ptx::tmem_ld_32x32b_x16(taddr, r);
          ptx::tmem_wait_ld();
          if (valid) {
            for (int g8 = 0; g8 < ncols; g8 += 8) {
              float v[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                float t = r16(__uint_as_float(r[g8 + j]) + sBias[cc + g8 + j]);
                if (a.act == kActRelu) {
                  t = fmaxf(t, 0.f);
                } else if (a.act == kActSilu) {
                  const float sg2 = r16(1.f / (1.f + __expf(-t)));
                  t = r16(t * sg2);
                }
                v[j] = t;
              }
              if (a.add1) {
                float ad[8];
                unpack8(*reinterpret_cast<const uint4*>(a.add1 + obase + cc + g8), ad);
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = r16(v[j] + ad[j]);
              }
              if (a.add2) {
                float ad[8];
                unpack8(*reinterpret_cast<const uint4*>(a.add2 + obase + cc + g8), ad);
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = r16(v[j] + ad[j]);
              }
              *reinterpret_cast<uint4*>(a.out + obase + cc + g8) = pack8(v);
            }
          }
        }
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(&acce[acc]));
        ++acc_cnt;
      }
    }
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
// Host side
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
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

int layout_for(int cw) { return cw == 64 ? 2 : (cw == 32 ? 4 : 6); }
CUtensorMapSwizzle swizzle_for(int cw) {
  return cw == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : (cw == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
}
int round_up(int v, int a) { return (v + a - 1) / a * a; }

void make_chunks(int C, ConvTcWeights* w) {
  int c = 0, n = 0;
  while (c < C) {
    const int rem = C - c;
    const int cw = rem >= 64 ? 64 : (rem >= 32 ? 32 : 16);
    ConvTcChunk& k = w->chunk[n++];
    k.c0 = c;
    k.cw = cw;
    k.rowbytes = cw * 2;
    k.layout = layout_for(cw);
    k.area = round_up(136 * k.rowbytes, 1024);
    c += cw;
  }
  w->nchunks = n;
  int off = 0;
  for (int i = 0; i < n; ++i) {
    w->chunk[i].slot_off = off;
    off += w->chunk[i].area;
  }
}

// Byte position of element (row m, channel k) inside one swizzled K-major block.
// Rows are `rb` bytes; 16-byte granule j of row m is stored at granule j ^ phase(m),
// where the phase is taken from address bits 7.. of the row (the 128B/64B/32B swizzle
// patterns repeat every 1024/512/256 bytes).
size_t swz_offset(int m, int k, int rb) {
  const size_t row = static_cast<size_t>(m) * rb;
  const int j = (k * 2) / 16;
  const int e = (k * 2) % 16;
  int phase;
  if (rb == 128) phase = m & 7;
  else if (rb == 64) phase = (m >> 1) & 3;
  else phase = (m >> 2) & 1;
  return row + static_cast<size_t>((j ^ phase) * 16 + e);
}

}  // namespace

bool conv_tc_supported(int C, int M, std::string* why) {
  // Three input-row slots of C channels plus the weights must fit in shared memory:
  // up to two 64-channel chunks per pixel row.
  if (C % 16 != 0 || C > 128) {
    if (why) *why = "tensor-core conv needs C % 16 == 0 and C <= 128";
    return false;
  }
  if (M % 16 != 0 || M > 256) {
    if (why) *why = "tensor-core conv needs M % 16 == 0 and M <= 256";
    return false;
  }
  return true;
}

std::vector<uint8_t> conv_tc_pack_host(const uint16_t* w_oihw, int C, int M, ConvTcWeights* L) {
  make_chunks(C, L);
  L->C = C;
  L->M = M;
  long long off = 0;
  for (int t = 0; t < 9; ++t)
    for (int k = 0; k < L->nchunks; ++k) {
      L->gofs[t * L->nchunks + k] = off;
      off += static_cast<long long>(M) * L->chunk[k].rowbytes;
    }
  std::vector<uint8_t> img(static_cast<size_t>(off), 0);
  for (int t = 0; t < 9; ++t) {
    for (int k = 0; k < L->nchunks; ++k) {
      const ConvTcChunk& ch = L->chunk[k];
      uint8_t* blk = img.data() + L->gofs[t * L->nchunks + k];
      for (int m = 0; m < M; ++m)
        for (int kk = 0; kk < ch.cw; ++kk) {
          const int c = ch.c0 + kk;
          const uint16_t v = w_oihw[(static_cast<size_t>(m) * C + c) * 9 + t];
          std::memcpy(blk + swz_offset(m, kk, ch.rowbytes), &v, 2);
        }
    }
  }
  L->wpack_bytes = img.size();
  return img;
}

cudaError_t conv_tc_upload(const uint16_t* w_oihw, const float* bias, int C, int M, ConvTcWeights* out) {
  std::vector<uint8_t> img = conv_tc_pack_host(w_oihw, C, M, out);
  cudaError_t e = cudaMalloc(&out->wpack, img.size());
  if (e != cudaSuccess) return e;
  e = cudaMemcpy(out->wpack, img.data(), img.size(), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return e;
  std::vector<float> b(M, 0.f);
  if (bias) std::memcpy(b.data(), bias, sizeof(float) * M);
  e = cudaMalloc(&out->bias, sizeof(float) * M);
  if (e != cudaSuccess) return e;
  return cudaMemcpy(out->bias, b.data(), sizeof(float) * M, cudaMemcpyHostToDevice);
}

void conv_tc_free(ConvTcWeights* w) {
  if (w->wpack) cudaFree(w->wpack);
  if (w->bias) cudaFree(w->bias);
  w->wpack = nullptr;
  w->bias = nullptr;
}

bool conv_tc_plan(const ConvTcWeights* w, const __half* in, int H, int W, int num_sms, ConvTcPlan* P,
                  std::string* err) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) {
    if (err) *err = "cuTensorMapEncodeTiled is unavailable from the CUDA driver";
    return false;
  }
  if ((reinterpret_cast<uintptr_t>(in) & 15u) != 0) {
    if (err) *err = "tensor-core conv input must be 16-byte aligned";
    return false;
  }
  P->w = w;
  P->H = H;
  P->W = W;
  int slot_bytes = 0;
  for (int k = 0; k < w->nchunks; ++k) slot_bytes += w->chunk[k].area;
  P->slot_bytes = slot_bytes;
  const int fixed = 1024 /*align slack*/ + 256 * 4 /*bias*/ + 256 /*barriers + flags*/;
  // Largest channel slice (divisor of M, multiple of 16) whose weights and >= 4 row
  // slots fit in shared memory; 3 slots is the functional minimum.
  int chosen = 0, slots = 0, wbytes_chosen = 0;
  for (int nsplit = 1; nsplit <= w->M / 16 && !chosen; ++nsplit) {
    if (w->M % nsplit) continue;
    const int MT = w->M / nsplit;
    if (MT % 16) continue;
    int wb = 0;
    for (int t = 0; t < 9; ++t)
      for (int k = 0; k < w->nchunks; ++k) wb += round_up(MT * w->chunk[k].rowbytes, 1024);
    for (int s = 4; s >= 3; --s) {
      if (wb + s * slot_bytes + fixed <= kSmemLimit) {
        chosen = MT;
        slots = s;
        wbytes_chosen = wb;
        break;
      }
    }
  }
  if (!chosen) {
    if (err) *err = "tensor-core conv: weights and row slots do not fit in shared memory";
    return false;
  }
  P->MT = chosen;
  P->n_msplit = w->M / chosen;
  P->nslots = slots;
  P->w_smem_bytes = wbytes_chosen;
  int off = 0;
  for (int t = 0; t < 9; ++t)
    for (int k = 0; k < w->nchunks; ++k) {
      P->wofs[t * w->nchunks + k] = off;
      off += round_up(chosen * w->chunk[k].rowbytes, 1024);
    }
  P->smem_bytes = static_cast<size_t>(wbytes_chosen + slots * slot_bytes + fixed);
  P->acc_stride = round_up(chosen, 32);
  P->nacc = (4 * P->acc_stride <= 512) ? 4 : 2;
  int cols = 32;
  while (cols < P->nacc * P->acc_stride) cols *= 2;
  P->tmem_cols = cols;
  const long long n_strips = (W + kTcTilePx - 1) / kTcTilePx;
  const long long rows_total = n_strips * H;
  long long gx = std::max(1, num_sms / P->n_msplit);
  if (gx > rows_total) gx = rows_total;
  P->grid_x = static_cast<int>(gx);

  const int C = w->C;
  for (int k = 0; k < w->nchunks; ++k) {
    const ConvTcChunk& ch = w->chunk[k];
    cuuint64_t gdim[3] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(W), static_cast<cuuint64_t>(H)};
    cuuint64_t gstride[2] = {static_cast<cuuint64_t>(C) * 2, static_cast<cuuint64_t>(W) * C * 2};
    cuuint32_t box[3] = {static_cast<cuuint32_t>(ch.cw), static_cast<cuuint32_t>(kTcBoxPx), 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(&P->maps[k], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(in), gdim, gstride, box,
                     estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_for(ch.cw), CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      if (err) *err = "cuTensorMapEncodeTiled failed (code " + std::to_string(static_cast<int>(r)) + ")";
      return false;
    }
  }
  return true;
}

cudaError_t conv_tc_launch(const ConvTcPlan& P, const __half* add1, const __half* add2, __half* out, int act,
                           uint32_t* status, cudaStream_t stream, int desc_base_mode) {
  const ConvTcWeights* w = P.w;
  ConvTcArgs a;
  std::memset(&a, 0, sizeof(a));
  for (int k = 0; k < w->nchunks; ++k) a.maps[k] = P.maps[k];
  a.wpack = static_cast<const uint8_t*>(w->wpack);
  a.bias = w->bias;
  a.add1 = add1;
  a.add2 = add2;
  a.out = out;
  a.status = status;
  for (int i = 0; i < 9 * w->nchunks; ++i) {
    a.gofs[i] = w->gofs[i];
    a.wofs[i] = P.wofs[i];
  }
  a.H = P.H;
  a.W = P.W;
  a.M = w->M;
  a.MT = P.MT;
  a.nchunks = w->nchunks;
  int tx = 0;
  for (int k = 0; k < w->nchunks; ++k) {
    a.rowbytes[k] = w->chunk[k].rowbytes;
    a.layout[k] = w->chunk[k].layout;
    a.kblocks[k] = w->chunk[k].cw / 16;
    a.c0[k] = w->chunk[k].c0;
    a.slot_off[k] = w->chunk[k].slot_off;
    tx += w->chunk[k].rowbytes * kTcBoxPx;
  }
  a.slot_bytes = P.slot_bytes;
  a.slot_tx = tx;
  a.nslots = P.nslots;
  a.w_smem_bytes = P.w_smem_bytes;
  a.n_strips = (P.W + kTcTilePx - 1) / kTcTilePx;
  a.rows_total = static_cast<long long>(a.n_strips) * P.H;
  a.act = act;
  a.desc_base_mode = desc_base_mode;
  a.nacc = P.nacc;
  a.acc_stride = P.acc_stride;
  a.tmem_cols = static_cast<uint32_t>(P.tmem_cols);

  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(conv3x3_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  dim3 grid(P.grid_x, P.n_msplit);
  conv3x3_tc_kernel<<<grid, kThreads, P.smem_bytes, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace ah
