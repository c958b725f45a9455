// Host side of the tcgen05 implicit-GEMM 3x3 convolution: weight packing into the swizzled
// K-major blocks the MMA reads, the per-frame launch plan (shared-memory layout, row-slot
// ring depth, channel slicing, TMEM ring, tensor maps) and the launch. The device code and
// its design notes are in conv_tc_kernel.cuh; its instantiations are spread over
// conv_tc_c*.cu (one file per input-channel count) so they compile in parallel.

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <unordered_set>

#include "conv_tc_kernel.cuh"

namespace ah {

using namespace tck;

namespace {

// Failure-path test hook (ah_test_set_conv_fault_hook): 0 = off.
std::atomic<int> g_test_wait_ms{0};
std::atomic<int> g_test_stall_row{-1};

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

// kx-in-N tail: two CTAs per SM (four row pipelines), two input slots per pipeline. Measured
// on B200 (R8F64 tail, 1080p, CUDA events in the frame graph): 2 slots 0.0607 ms, 3 slots
// 0.0624 ms, one CTA per SM with 6 slots per pipeline 0.0646 ms; deeper rings do not help
// a tail whose rows are bound by their per-row MMA and epilogue chains.
constexpr bool kKxnTwoCtas = true;
constexpr int kKxnMaxSlots = 2;

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

bool encode(EncodeTiledFn enc, CUtensorMap* map, const void* base, int C, int W, int H, int box_c, int box_px,
            std::string* err) {
  cuuint64_t gdim[3] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(W), static_cast<cuuint64_t>(H)};
  cuuint64_t gstride[2] = {static_cast<cuuint64_t>(C) * 2, static_cast<cuuint64_t>(W) * C * 2};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box_c), static_cast<cuuint32_t>(box_px), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), gdim, gstride, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_for(box_c), CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    if (err) *err = "cuTensorMapEncodeTiled failed (code " + std::to_string(static_cast<int>(r)) + ")";
    return false;
  }
  return true;
}

}  // namespace

bool encode_nhwc_map(CUtensorMap* map, const void* base, int C, int W, int H, int box_c, int box_px,
                     std::string* err) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) {
    if (err) *err = "cuTensorMapEncodeTiled is unavailable from the CUDA driver";
    return false;
  }
  return encode(enc, map, base, C, W, H, box_c, box_px, err);
}

bool conv_tc_supported(int C, int M, std::string* why) {
  // Three input-row slots of C channels plus the weights must fit in shared memory:
  // up to two 64-channel chunks per pixel row.
  if (C % 16 != 0 || C > 128) {
    if (why) *why = "tensor-core conv needs C % 16 == 0 and C <= 128";
    return false;
  }
  if (M < 1 || M > 256) {
    if (why) *why = "tensor-core conv needs 1 <= M <= 256";
    return false;
  }
  return true;
}

namespace {

int slot_bytes_of(const ConvTcWeights* w) {
  int s = 0;
  for (int k = 0; k < w->nchunks; ++k) s += w->chunk[k].area;
  return s;
}

// Shared memory of a plan: weights + row slots + ones/bias tiles + staging + tail.
// Staging bytes of one epilogue warp: the standard kernel's 8 warps take alternate 32-channel
// groups; the vertical-window kernel's 4 warps per pipe take every group of their quarter.
int stage_per_warp_of(int MT, bool vert, int mode) {
  if (mode != 0) return 0;
  const int ngroups = (MT + 31) / 32;
  return (vert ? ngroups : (ngroups + 1) / 2) * kStageTile;
}

// Shared memory of a plan: weights + row slots (per pipe: two pipes in the vertical-window
// kernel) + ones/bias tiles + staging + tail.
int smem_need(const ConvTcWeights* w, int MT, bool vert, int mode, int slots) {
  int wb = 0;
  for (int b = 0; b < (vert ? 3 : 9); ++b)
    for (int k = 0; k < w->nchunks; ++k) wb += round_up((vert ? 3 : 1) * MT * w->chunk[k].rowbytes, 1024);
  const int pipes = vert ? 2 : 1;
  return wb + pipes * slots * slot_bytes_of(w) + 4096 + round_up(MT * 32, 1024) +
         kEpiWarps * stage_per_warp_of(MT, vert, mode) + kTailBytes + 1024;
}

}  // namespace

size_t conv_tc_pack_layout(int C, int M, ConvTcWeights* L) {
  make_chunks(C, L);
  L->C = C;
  L->M = M;
  L->Mpad = round_up(M, 16);
  // The vertical-window formulation takes slices of vmt = 16, 32, 48 or 64 output channels
  // (3 * vmt <= 256 columns per MMA; a ring of four or more vmt-column chunks per pipe):
  // the whole Mpad when it is one of those, else 64- or 48-channel slices, one per CTA row
  // of the grid. The slice's weights and 3 input-row slots per pipe (2 when the channels
  // are sliced: the standard form would slice them too) must fit in shared memory.
  const int Mp = L->Mpad;
  int vmt = 0;
  if (Mp == 16 || Mp == 32 || Mp == 48 || Mp == 64) vmt = Mp;
  else if (Mp % 64 == 0) vmt = 64;
  else if (Mp % 48 == 0) vmt = 48;
  const int min_slots = (vmt && Mp > vmt) ? 2 : 3;
  L->vert = (vmt && smem_need(L, vmt, true, 0, min_slots) <= kSmemLimit) ? 1 : 0;
  L->vmt = L->vert ? vmt : 0;
  const int nblk = L->vert ? 3 : 9;
  const int rows = L->vert ? 3 * Mp : Mp;
  long long off = 0;
  for (int b = 0; b < nblk; ++b)
    for (int k = 0; k < L->nchunks; ++k) {
      L->gofs[b * L->nchunks + k] = off;
      off += static_cast<long long>(rows) * L->chunk[k].rowbytes;
    }
  // Four-channel convs (the 2x DepthToSpace tails of luma models) also get the kx-in-N
  // blocks: 3 x 16 rows per chunk.
  L->kxn = (L->vert && M == 4 && Mp == 16 && L->vmt == 16) ? 1 : 0;
  for (int k = 0; k < L->nchunks; ++k) {
    L->kxn_gofs[k] = L->kxn ? off : 0;
    if (L->kxn) off += 3LL * 16 * L->chunk[k].rowbytes;
  }
  L->wpack_bytes = static_cast<size_t>(off);
  return L->wpack_bytes;
}

void conv_tc_pack_into(const uint16_t* w_oihw, const ConvTcWeights& L, uint8_t* img) {
  std::memset(img, 0, L.wpack_bytes);
  const int C = L.C, M = L.M, Mp = L.Mpad;
  for (int b = 0; b < (L.vert ? 3 : 9); ++b) {
    for (int k = 0; k < L.nchunks; ++k) {
      const ConvTcChunk& ch = L.chunk[k];
      uint8_t* blk = img + L.gofs[b * L.nchunks + k];
      // standard: block b = tap, row = m; vertical: block b = kx, row = slice * 3 vmt +
      // ky * vmt + (m - slice * vmt) (rows of the padding channels m >= M stay zero)
      const int vmt = L.vmt;
      for (int r = 0; r < (L.vert ? 3 * Mp : M); ++r) {
        int m = r, tap = b;
        if (L.vert) {
          const int sl = r / (3 * vmt), rr = r - sl * 3 * vmt;
          m = sl * vmt + rr % vmt;
          tap = (rr / vmt) * 3 + b;
        }
        if (m >= M) continue;
        for (int kk = 0; kk < ch.cw; ++kk) {
          const int c = ch.c0 + kk;
          const uint16_t v = w_oihw[(static_cast<size_t>(m) * C + c) * 9 + tap];
          std::memcpy(blk + swz_granule(r, (kk * 2) / 16, ch.rowbytes) + (kk * 2) % 16, &v, 2);
        }
      }
    }
  }
  if (!L.kxn) return;
  // kx-in-N blocks: row ky * 16 + kx * 4 + m holds w[m][.][ky][kx] (rows 12..15 of each
  // kernel row stay zero).
  for (int k = 0; k < L.nchunks; ++k) {
    const ConvTcChunk& ch = L.chunk[k];
    uint8_t* blk = img + L.kxn_gofs[k];
    for (int ky = 0; ky < 3; ++ky)
      for (int kx = 0; kx < 3; ++kx)
        for (int m = 0; m < M; ++m) {
          const int r = ky * 16 + kx * 4 + m;
          for (int kk = 0; kk < ch.cw; ++kk) {
            const uint16_t v = w_oihw[(static_cast<size_t>(m) * C + ch.c0 + kk) * 9 + ky * 3 + kx];
            std::memcpy(blk + swz_granule(r, (kk * 2) / 16, ch.rowbytes) + (kk * 2) % 16, &v, 2);
          }
        }
  }
}

std::vector<uint8_t> conv_tc_pack_host(const uint16_t* w_oihw, int C, int M, ConvTcWeights* L) {
  std::vector<uint8_t> img(conv_tc_pack_layout(C, M, L));
  conv_tc_pack_into(w_oihw, *L, img.data());
  return img;
}

cudaError_t conv_tc_upload(const uint16_t* w_oihw, const float* bias, int C, int M, ConvTcWeights* out) {
  std::vector<uint8_t> img = conv_tc_pack_host(w_oihw, C, M, out);
  cudaError_t e = cudaMalloc(&out->wpack, img.size());
  if (e != cudaSuccess) return e;
  e = cudaMemcpy(out->wpack, img.data(), img.size(), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return e;
  std::vector<float> b(out->Mpad, 0.f);
  if (bias) std::memcpy(b.data(), bias, sizeof(float) * M);
  e = cudaMalloc(&out->bias, sizeof(float) * out->Mpad);
  if (e != cudaSuccess) return e;
  return cudaMemcpy(out->bias, b.data(), sizeof(float) * out->Mpad, cudaMemcpyHostToDevice);
}

void conv_tc_free(ConvTcWeights* w) {
  if (w->wpack) cudaFree(w->wpack);
  if (w->bias) cudaFree(w->bias);
  w->wpack = nullptr;
  w->bias = nullptr;
}

bool conv_tc_plan(const ConvTcWeights* w, const __half* in, int H, int W, const ConvTcOut& out, int num_sms,
                  ConvTcPlan* P, std::string* err) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) {
    if (err) *err = "cuTensorMapEncodeTiled is unavailable from the CUDA driver";
    return false;
  }
  if ((reinterpret_cast<uintptr_t>(in) & 15u) != 0 ||
      (out.mode == 0 && (reinterpret_cast<uintptr_t>(out.ptr) & 15u) != 0)) {
    if (err) *err = "tensor-core conv buffers must be 16-byte aligned";
    return false;
  }
  if (out.mode == 0 && w->M != w->Mpad) {
    if (err) *err = "tensor-core conv NHWC output needs M % 16 == 0";
    return false;
  }
  P->w = w;
  P->H = H;
  P->W = W;
  P->out = out;
  P->kxn = 0;
  const int slot_bytes = slot_bytes_of(w);
  P->slot_bytes = slot_bytes;
  const bool vert = w->vert != 0;
  int chosen = 0, slots = 0;
  bool dual = false;  // two CTAs per SM
  if (vert) {
    // One channel slice per CTA row of the grid; deepest input-row ring that fits.
    const int min_slots = w->Mpad > w->vmt ? 2 : 3;
    // The 2x DepthToSpace tail (narrow N, little tensor work per row) is bound by its
    // per-row MMA issue and epilogue chains, not by loads: it runs two CTAs per SM, each
    // with two input slots per pipe and half of the tensor memory.
    const bool dts_tail =
        out.mode == 1 && out.dts_b == 2 && (out.nchw || w->M == 4) && w->M % 4 == 0 && w->Mpad == 16;
    // The kx-in-N form of a four-channel tail, for a launch without residual operands
    // (ARTHIP_TAIL_KXN=0 keeps the three-kx form; read when the plan is built, never at
    // launch). Its slots are 128 rows and its weights one block per chunk, so it fits
    // twice per SM up to C = 96.
    const char* v = std::getenv("ARTHIP_TAIL_KXN");
    if (dts_tail && w->kxn && out.adds == 0 && !(v && *v == '0')) {
      int kslot = 0, kw = 0;
      for (int k = 0; k < w->nchunks; ++k) {
        kslot += kTcTilePx * w->chunk[k].rowbytes;
        kw += round_up(3 * w->vmt * w->chunk[k].rowbytes, 1024);
      }
      const int limit = kKxnTwoCtas ? kSmemPerSm / 2 - 1024 : kSmemLimit;
      for (int s2 = kKxnMaxSlots; s2 >= 2 && !chosen; --s2)
        if (kw + 2 * s2 * kslot + 4096 + round_up(w->vmt * 32, 1024) + kTailBytes + 1024 <= limit) {
          P->kxn = 1;
          P->slot_bytes = kslot;
          chosen = w->vmt;
          slots = s2;
          dual = kKxnTwoCtas;
        }
    }
    if (!chosen) {
      dual = dts_tail && smem_need(w, w->vmt, true, out.mode, 2) <= kSmemPerSm / 2 - 1024;
      if (dual) {
        chosen = w->vmt;
        slots = 2;
      }
    }
    for (int s = kMaxSlots; s >= min_slots && !chosen; --s)
      if (smem_need(w, w->vmt, true, out.mode, s) <= kSmemLimit) {
        chosen = w->vmt;
        slots = s;
      }
  } else {
    // Largest channel slice (divisor of Mpad, multiple of 16) whose weights, bias tile,
    // staging tiles and >= 4 input-row slots fit in shared memory (3 is the minimum).
    for (int nsplit = 1; nsplit <= w->Mpad / 16 && !chosen; ++nsplit) {
      if (w->Mpad % nsplit) continue;
      const int MT = w->Mpad / nsplit;
      if (MT % 16) continue;
      bool can_split = false;
      for (int ns = nsplit + 1; ns <= w->Mpad / 16; ++ns)
        if (w->Mpad % ns == 0 && (w->Mpad / ns) % 16 == 0) can_split = true;
      for (int s = kMaxSlots; s >= 3; --s) {
        if (smem_need(w, MT, false, out.mode, s) <= kSmemLimit) {
          if (s < 4 && can_split) break;  // rather split the channels than run a 3-slot ring
          chosen = MT;
          slots = s;
          break;
        }
      }
    }
  }
  if (!chosen) {
    if (err) *err = "tensor-core conv: weights and row slots do not fit in shared memory";
    return false;
  }
  P->vert = vert ? 1 : 0;
  P->MT = chosen;
  P->n_msplit = w->Mpad / chosen;
  P->nslots = slots;
  int off = 0;
  for (int b = 0; b < (P->kxn ? 1 : (vert ? 3 : 9)); ++b)
    for (int k = 0; k < w->nchunks; ++k) {
      P->wofs[b * w->nchunks + k] = off;
      off += round_up((vert ? 3 : 1) * chosen * w->chunk[k].rowbytes, 1024);
    }
  P->w_smem_bytes = off;
  off += (vert ? 2 : 1) * slots * P->slot_bytes;
  P->ones_off = off;
  off += 4096;
  P->biasb_off = off;
  off += round_up(chosen * 32, 1024);
  P->stage_off = off;
  P->stage_per_warp = stage_per_warp_of(chosen, vert, out.mode);
  off += kEpiWarps * P->stage_per_warp;
  P->smem_bytes = static_cast<size_t>(off) + kTailBytes + 1024;
  if (vert) {
    // Two pipes, each with half of the CTA's TMEM columns (all 512, or 256 with two CTAs
    // per SM) as a ring of chunks of M columns (a power of two, at most kMaxAcc of them),
    // one per output row in flight.
    P->tmem_cols = dual ? 256 : 512;
    P->acc_stride = chosen;
    int nacc = std::min(P->tmem_cols / 2 / chosen, kMaxAcc);
    while (nacc & (nacc - 1)) nacc &= nacc - 1;
    P->nacc = nacc;
  } else {
    P->acc_stride = round_up(chosen, 32);
    P->nacc = (4 * P->acc_stride <= 512) ? 4 : 2;
    int cols = 32;
    while (cols < P->nacc * P->acc_stride) cols *= 2;
    P->tmem_cols = cols;
  }
  const long long n_strips = (W + kTcTilePx - 1) / kTcTilePx;
  const long long rows_total = n_strips * H;
  long long gx = std::max(1, (dual ? 2 : 1) * num_sms / P->n_msplit);
  if (gx > rows_total) gx = rows_total;
  P->grid_x = static_cast<int>(gx);

  // (the kx-in-N tail loads 32-pixel sub-tiles)
  for (int k = 0; k < w->nchunks; ++k)
    if (!encode(enc, &P->maps[k], in, w->C, W, H, w->chunk[k].cw, P->kxn ? kKxnSub : kTcBoxPx, err)) return false;
  if (out.mode == 0) {
    if (chosen >= 32 && !encode(enc, &P->out_map32, out.ptr, w->M, W, H, 32, 32, err)) return false;
    if (chosen % 32 == 16 && !encode(enc, &P->out_map16, out.ptr, w->M, W, H, 16, 32, err)) return false;
  }
  // Opt every output variant of this (C, formulation) into the large shared-memory carve-out
  // now, outside any stream capture (the variant is chosen at launch from act and adds).
  static std::mutex mu;
  static std::unordered_set<const void*> attr_set;
  std::lock_guard<std::mutex> lock(mu);
  for (int v = 0; v < kVariants; ++v) {
    KernelFn fn = kernel_for(w->C, vert, v);
    if (attr_set.count(reinterpret_cast<const void*>(fn))) continue;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    if (e != cudaSuccess) {
      if (err) *err = std::string("cudaFuncSetAttribute failed: ") + cudaGetErrorString(e);
      return false;
    }
    attr_set.insert(reinterpret_cast<const void*>(fn));
  }
  return true;
}

void conv_tc_set_test_hook(int wait_limit_ms, int stall_row) {
  const bool on = wait_limit_ms > 0 && wait_limit_ms <= 4000 && stall_row >= 0;
  g_test_stall_row.store(on ? stall_row : -1, std::memory_order_relaxed);
  g_test_wait_ms.store(on ? wait_limit_ms : 0, std::memory_order_relaxed);
}

cudaError_t conv_tc_launch(const ConvTcPlan& P, const __half* add1, const __half* add2, int act, uint32_t* status,
                           cudaStream_t stream) {
  const ConvTcWeights* w = P.w;
  ConvTcArgs a;
  std::memset(&a, 0, sizeof(a));
  for (int k = 0; k < w->nchunks; ++k) a.maps[k] = P.maps[k];
  a.out_map32 = P.out_map32;
  a.out_map16 = P.out_map16;
  a.wpack = static_cast<const uint8_t*>(w->wpack);
  a.bias = w->bias;
  // The kernel takes a second residual operand only together with a first one.
  a.add1 = add1 ? add1 : add2;
  a.add2 = add1 ? add2 : nullptr;
  // In place: when the NHWC output buffer is the last residual operand (the engine aliases
  // them once that operand is dead), the epilogue does not load it; the tile stores become
  // TMA reduce-adds, so L2 adds the operand: fp16(r + t) == fp16(t + r), the graph's Add.
  const __half* last = a.add2 ? a.add2 : a.add1;
  if (P.out.mode == 0 && last && static_cast<const void*>(last) == P.out.ptr) {
    a.reduce_out = 1;
    if (a.add2) a.add2 = nullptr;
    else a.add1 = nullptr;
  }
  // The two-pipeline kernel TMA-loads the first remaining operand into its staging tiles
  // (same tile geometry as the output stores); if a map cannot be made, it loads per lane.
  if (P.vert && P.out.mode == 0 && a.add1) {
    EncodeTiledFn enc = get_encode_fn();
    bool good = enc != nullptr;
    if (good && P.MT >= 32) good = encode(enc, &a.res_map32, a.add1, w->M, P.W, P.H, 32, 32, nullptr);
    if (good && P.MT % 32 == 16) good = encode(enc, &a.res_map16, a.add1, w->M, P.W, P.H, 16, 32, nullptr);
    a.res_tma = good ? 1 : 0;
  }
  a.status = status;
  a.out = P.out;
  for (int i = 0; i < 9 * w->nchunks; ++i) {
    a.gofs[i] = w->gofs[i];
    a.wofs[i] = P.wofs[i];
  }
  a.H = P.H;
  a.W = P.W;
  a.M = w->M;
  a.Mpad = w->Mpad;
  a.MT = P.MT;
  int tx = 0;
  for (int k = 0; k < w->nchunks; ++k) {
    a.c0[k] = w->chunk[k].c0;
    a.slot_off[k] = w->chunk[k].slot_off;
    tx += w->chunk[k].rowbytes * (P.kxn ? kTcTilePx : kTcBoxPx);  // kx-in-N: 4 x 32-pixel sub-tiles
  }
  a.slot_bytes = P.slot_bytes;
  a.slot_tx = tx;
  a.nslots = P.nslots;
  a.w_smem_bytes = P.w_smem_bytes;
  a.ones_off = P.ones_off;
  a.biasb_off = P.biasb_off;
  a.stage_off = P.stage_off;
  a.stage_per_warp = P.stage_per_warp;
  // (the strips of the kx-in-N tail advance by kKxnStride pixels; set with its variant below)
  a.rows_total = static_cast<long long>((P.W + kTcTilePx - 1) / kTcTilePx) * P.H;
  a.act = act;
  a.nacc = P.nacc;
  a.acc_stride = P.acc_stride;
  a.tmem_cols = static_cast<uint32_t>(P.tmem_cols);
  // Pipeline waits are bounded (4 s). The failure-path test hook (off unless a test sets
  // it through ah_test_set_conv_fault_hook) shortens the bound and makes every CTA arm one
  // input row's slot without loading it, so the kernel must report a timed-out wait
  // through the status word and leave the context usable.
  const int hook_ms = g_test_wait_ms.load(std::memory_order_relaxed);
  a.wait_limit_ns = hook_ms > 0 ? static_cast<unsigned long long>(hook_ms) * 1000000ull : 4000000000ull;
  a.stall_row = hook_ms > 0 ? g_test_stall_row.load(std::memory_order_relaxed) : -1;
  // Output variant: NHWC with a compile-time activation, the 2x DepthToSpace tail (every
  // conv channel in one CTA's first 32-channel group, no residual; NCHW output, which for
  // one output channel is also the NHWC layout), or general stores.
  int variant = 4;
  if (P.out.mode == 0) {
    variant = act == kActRelu ? 1 : (act == kActSilu ? 2 : 0);
    // SiLU over 64-channel slices: the epilogue math is the bound, so eight epilogue warps
    // per pipe (one per lane quarter and channel group).
    if (variant == 2 && P.vert && P.MT == 64) variant = 5;
  } else if (P.out.dts_b == 2 && (P.out.nchw || w->M == 4) && !a.add1 && P.n_msplit == 1 && w->M % 4 == 0 &&
             w->M <= 16 && w->M <= P.MT) {
    variant = 3;
    if (P.kxn) {
      // kx-in-N tail: one weight block per chunk, strips of kKxnStride pixels
      variant = 6;
      for (int k = 0; k < w->nchunks; ++k) a.gofs[k] = w->kxn_gofs[k];
      a.rows_total = static_cast<long long>((P.W + kKxnStride - 1) / kKxnStride) * P.H;
    }
  }
  // A kx-in-N plan (tensor maps, slot layout) serves only that variant: it is built for
  // launches without residual operands.
  if (P.kxn && variant != 6) return cudaErrorInvalidValue;
  // Programmatic dependent launch: this kernel's set-up (barriers, TMEM, weights) overlaps
  // the previous kernel's last CTAs; it waits in hardware (griddepcontrol.wait) before it
  // reads the previous layers' activations or writes its output. ARTHIP_NO_PDL=1 turns it off.
  static const bool no_pdl = [] {
    const char* v = std::getenv("ARTHIP_NO_PDL");
    return v && *v == '1';
  }();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(P.grid_x, P.n_msplit);
  cfg.blockDim = dim3(P.vert ? (variant == 5 ? kThreads2W : kThreads2) : kThreads);
  cfg.dynamicSmemBytes = P.smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = no_pdl ? 0 : 1;
  return cudaLaunchKernelEx(&cfg, kernel_for(w->C, P.vert != 0, variant), a);
}

}  // namespace ah

namespace ah {
namespace tck {

KernelFn kernel_c16(bool vert, int variant);
KernelFn kernel_c32(bool vert, int variant);
KernelFn kernel_c48(bool vert, int variant);
KernelFn kernel_c64(bool vert, int variant);
KernelFn kernel_c80(bool vert, int variant);
KernelFn kernel_c96(bool vert, int variant);
KernelFn kernel_c112(bool vert, int variant);
KernelFn kernel_c128(bool vert, int variant);

KernelFn kernel_for(int C, bool vert, int variant) {
  switch (C) {
    case 16: return kernel_c16(vert, variant);
    case 32: return kernel_c32(vert, variant);
    case 48: return kernel_c48(vert, variant);
    case 64: return kernel_c64(vert, variant);
    case 80: return kernel_c80(vert, variant);
    case 96: return kernel_c96(vert, variant);
    case 112: return kernel_c112(vert, variant);
    default: return kernel_c128(vert, variant);
  }
}

}  // namespace tck
}  // namespace ah
