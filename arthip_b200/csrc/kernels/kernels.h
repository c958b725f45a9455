// Host-side launch interface of the device kernels (sm_100a).
//
// Tensors are fp16 NHWC ([H][W][C], batch 1) inside the engine; the graph boundary is
// NCHW in the model's IO dtype. Every launcher returns a cudaError_t from the launch.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace ah {

enum Act : int { kActNone = 0, kActRelu = 1, kActSilu = 2 };

#ifdef __CUDACC__
// Logistic sigmoid for the SiLU epilogues and the Sigmoid op, from the hardware exp2 and
// divide approximations (__expf, __fdividef: errors of a few fp32 ulp; 0 for very large
// -v). Every caller rounds the result to fp16 next, which absorbs that error except where
// the exact value lies within ~1e-6 of an fp16 rounding boundary (a one-ulp difference).
// The libm expf and IEEE division made the SiLU convs epilogue-bound.
__device__ __forceinline__ float sigmoid_fast(float v) { return __fdividef(1.f, 1.f + __expf(-v)); }
#endif

// ---------------------------------------------------------------------------
// tcgen05 implicit-GEMM 3x3 convolution (conv_tc.cu)
// ---------------------------------------------------------------------------
constexpr int kTcMaxChunks = 4;   // input channels <= 256
constexpr int kTcTilePx = 128;    // output pixels per MMA tile (one row segment)
constexpr int kTcBoxPx = 130;     // input pixels staged per row (tile + 1-pixel halo each side)

struct ConvTcChunk {
  int c0 = 0;        // first input channel of the chunk
  int cw = 0;        // channels in the chunk: 64, 32 or 16
  int rowbytes = 0;  // cw * 2 (one pixel row of the K-major operand)
  int layout = 0;    // smem descriptor layout code: 2 = 128B swizzle, 4 = 64B, 6 = 32B
  int area = 0;      // bytes of this chunk inside one input-row slot (1024-aligned)
  int slot_off = 0;  // offset of this chunk inside a slot
};

// Everything the kernel needs that depends only on (C, M, weights): built once per model.
struct ConvTcWeights {
  int C = 0, M = 0;
  int Mpad = 0;                // M rounded up to 16 (zero weights and bias in the padding)
  // Vertical-window packing: the output channels form slices of vmt = 16, 32, 48 or 64
  // (one slice per CTA row of the grid), and one block per (kx, chunk) holds, slice after
  // slice, the three kernel rows ky stacked along N (3 * vmt rows per slice), so one MMA of
  // N = 3 * vmt serves the three output rows an input row feeds. Otherwise one block of
  // Mpad rows per (tap, chunk).
  int vert = 0;
  int vmt = 0;
  // kx-in-N tail blocks (M == 4, vertical window): one block per chunk after the blocks
  // above, rows ky * 16 + kx * 4 + m (12 of each 16 used), for the 2x DepthToSpace tail.
  int kxn = 0;
  long long kxn_gofs[kTcMaxChunks] = {};
  int nchunks = 0;
  ConvTcChunk chunk[kTcMaxChunks];
  void* wpack = nullptr;       // device: swizzled K-major weight blocks (see vert)
  size_t wpack_bytes = 0;
  long long gofs[9 * kTcMaxChunks] = {};  // byte offset of each (tap, chunk) block
  float* bias = nullptr;       // device: Mpad fp32 (fp16-rounded values)
};

// Output of a tensor-core conv launch.
struct ConvTcOut {
  void* ptr = nullptr;
  // 0: NHWC fp16 [H][W][M], written with TMA stores from a swizzled staging tile.
  // 1: per-element stores: DepthToSpace (DCR, block dts_b; 1 = none), optional clip,
  //    fp16 or fp32, NCHW (graph boundary) or NHWC. Used by narrow tails.
  int mode = 0;
  int dts_b = 1;
  int nchw = 0;
  int fp32 = 0;
  int clip = 0;
  float clip_lo = 0.f, clip_hi = 0.f;
  // Residual operands the launches of this plan pass (-1: not known). A 2x DepthToSpace
  // tail of four channels without any takes the kx-in-N form.
  int adds = -1;
};

// Per (layer, buffers, frame size) launch plan.
struct ConvTcPlan {
  const ConvTcWeights* w = nullptr;
  int H = 0, W = 0;
  int MT = 0, n_msplit = 1;    // output channels per CTA and number of channel slices
  int nslots = 0;
  int slot_bytes = 0;
  int wofs[9 * kTcMaxChunks] = {};  // smem offset of each (tap, chunk) weight block
  int w_smem_bytes = 0;
  int ones_off = 0, biasb_off = 0, stage_off = 0, stage_per_warp = 0;
  size_t smem_bytes = 0;
  int nacc = 0, acc_stride = 0, tmem_cols = 0;
  int vert = 0;                // vertical window (two row pipelines per CTA; weights packed accordingly)
  int kxn = 0;                 // the kx-in-N 2x DepthToSpace tail (strips of 126 pixels)
  int grid_x = 0;
  ConvTcOut out;
  CUtensorMap maps[kTcMaxChunks];
  CUtensorMap out_map32, out_map16;
};

// Tensor map over an NHWC fp16 tensor [H][W][C] with a {box_c, box_px, 1} box, swizzled to
// match a box_c * 2-byte row (box_c 64: 128B, 32: 64B, 16: 32B swizzle).
bool encode_nhwc_map(CUtensorMap* map, const void* base, int C, int W, int H, int box_c, int box_px,
                     std::string* err);
// Returns true when the tensor-core kernel covers (C, M); otherwise fills `why`.
bool conv_tc_supported(int C, int M, std::string* why);
// Packs fp16 weights OIHW [M][C][3][3] (host, as fp16 bits) and fp32 bias into device memory.
cudaError_t conv_tc_upload(const uint16_t* w_oihw_f16, const float* bias_or_null, int C, int M,
                           ConvTcWeights* out);
void conv_tc_free(ConvTcWeights* w);
// Host-only packing: the layout (chunks, block offsets, formulation) and its byte size,
// then the swizzled image into a caller buffer of that size, or into a new vector.
size_t conv_tc_pack_layout(int C, int M, ConvTcWeights* layout);
void conv_tc_pack_into(const uint16_t* w_oihw_f16, const ConvTcWeights& layout, uint8_t* img);
std::vector<uint8_t> conv_tc_pack_host(const uint16_t* w_oihw_f16, int C, int M, ConvTcWeights* layout);
// Builds the per-frame plan (tensor maps over `in` and, for mode 0, `out.ptr`).
// Fails with a message when the tiles cannot fit in shared memory.
bool conv_tc_plan(const ConvTcWeights* w, const __half* in, int H, int W, const ConvTcOut& out, int num_sms,
                  ConvTcPlan* plan, std::string* err);
cudaError_t conv_tc_launch(const ConvTcPlan& plan, const __half* add1, const __half* add2, int act,
                           uint32_t* status, cudaStream_t stream);
// Failure-path test hook for later launches (process-wide): wait bound in ms (1..4000) and
// the CTA-relative input row whose slot every CTA arms without loading it. Any other value
// turns it off (the default: 4 s bound, no stalled row).
void conv_tc_set_test_hook(int wait_limit_ms, int stall_row);

// ---------------------------------------------------------------------------
// Two-SM (cta_group::2) vertical-window tensor-core convolution, 64 -> 64 channels, NHWC
// fp16 output with the fused activation and up to two residual adds (conv_tc_pair.cu).
// ---------------------------------------------------------------------------
struct PairWeights {
  void* wpack = nullptr;  // device: [2 CTA ranks][3 kx][320 rows][128 B] swizzled weight pieces
  float* bias = nullptr;  // device: 64 fp32
};
struct PairPlan {
  const PairWeights* w = nullptr;
  int H = 0, W = 0;
  __half* out = nullptr;
  long long rows_total = 0;  // (256-pixel strips) x H
  int grid_x = 0;            // 2 x clusters
  CUtensorMap in_map, out_map32;
};
bool pair_supported(int C, int M);
cudaError_t pair_upload(const uint16_t* w_oihw_f16, const float* bias_or_null, int C, int M, PairWeights* out);
void pair_free(PairWeights* w);
bool pair_plan(const PairWeights* w, const __half* in, int H, int W, __half* out, int num_sms, PairPlan* plan,
               std::string* err);
// out may be the last residual operand (in place: reduce-add stores, as conv_tc_launch).
cudaError_t pair_launch(const PairPlan& plan, const __half* add1, const __half* add2, int act, uint32_t* status,
                        cudaStream_t stream);

// ---------------------------------------------------------------------------
// Winograd F(2x2,3x3) tensor-core convolution, 64 -> 64 channels (conv_wino.cu): fp16
// transformed operands (the reference's numerics), opt-in through the engine's conv
// algorithm. NHWC fp16 output with the fused activation and up to two residual adds.
// ---------------------------------------------------------------------------
struct WinoWeights {
  void* upack = nullptr;   // device: U = G g G^T, [2 output halves][16 points][32 x 64] swizzled
  float* bias = nullptr;   // device: 64 fp32
};
struct WinoPlan {
  const WinoWeights* w = nullptr;
  int H = 0, W = 0;
  __half* out = nullptr;
  int units_x = 0;
  long long units = 0;
  int grid_x = 0;
  CUtensorMap in_map;
};
bool wino_supported(int C, int M);
cudaError_t wino_upload(const uint16_t* w_oihw_f16, const float* bias_or_null, int C, int M, WinoWeights* out);
void wino_free(WinoWeights* w);
bool wino_plan(const WinoWeights* w, const __half* in, int H, int W, __half* out, int num_sms, WinoPlan* plan,
               std::string* err);
// out may be the last residual operand (in place): each element is read before it is written.
cudaError_t wino_launch(const WinoPlan& plan, const __half* add1, const __half* add2, int act, uint32_t* status,
                        cudaStream_t stream);

// ---------------------------------------------------------------------------
// CUDA-core convolution for narrow layers (conv_simt.cu): C==1 heads, small M
// tails (with fused DepthToSpace / Clip / boundary layout), odd channel counts.
// ---------------------------------------------------------------------------
struct SimtOut {
  void* ptr = nullptr;
  int dts_b = 1;        // DepthToSpace block size (1 = none); DCR channel order
  int nchw = 0;         // 1: write [Cout][H*b][W*b] (graph boundary), 0: NHWC
  int fp32 = 0;         // 1: fp32 elements
  int clip = 0;
  float clip_lo = 0.f, clip_hi = 0.f;
};

struct SimtConvWeights {
  int C = 0, M = 0;
  float* w = nullptr;    // device: [tap][c][m] fp32 (values of the fp16 weights)
  float* bias = nullptr; // device: M fp32
  uint32_t* bfrag = nullptr;  // device: mma.sync B fragments of the tensor-core head (conv_head.cu)
};
cudaError_t simt_conv_upload(const uint16_t* w_oihw_f16, const float* bias_or_null, int C, int M,
                             SimtConvWeights* out);
void simt_conv_free(SimtConvWeights* w);
cudaError_t simt_conv_launch(const SimtConvWeights& w, const __half* in, int H, int W, const __half* add1,
                             const __half* add2, int act, const SimtOut& out, cudaStream_t stream);

// Tensor-core (mma.sync) head conv for C <= 4 input channels, M in {32, 64, 96, 128},
// plain NHWC fp16 output without residual adds (conv_head.cu). simt_conv_upload /
// simt_conv_launch use it when it applies.
bool head_mma_supported(int C, int M);
// (C == 1: the bias rides in the fragments, as the product of a constant 1 in K slot 12)
std::vector<uint32_t> head_mma_fragments(const uint16_t* w_oihw_f16, const float* bias_or_null, int C, int M);
cudaError_t head_mma_launch(const uint32_t* bfrag, const float* bias, int C, int M, const __half* in, int H, int W,
                            int act, __half* out, cudaStream_t s);

// ---------------------------------------------------------------------------
// Pointwise / layout kernels (pointwise.cu)
// ---------------------------------------------------------------------------
enum UnaryOp : int { kSigmoid = 0, kClip = 1, kRelu = 2 };
cudaError_t unary_launch(const __half* in, __half* out, size_t n, int op, float lo, float hi,
                         cudaStream_t s);
enum BinaryOp : int { kAdd = 0, kMul = 1 };
cudaError_t binary_launch(const __half* a, const __half* b, __half* out, size_t n, int op, cudaStream_t s);
// NHWC [H][W][Cout*b*b] -> DepthToSpace (DCR) -> SimtOut layout, optional clip.
cudaError_t dts_launch(const __half* in, int H, int W, int Cin, const SimtOut& out, cudaStream_t s);
// Boundary layout conversions. NCHW (fp16|fp32) -> NHWC fp16, and back.
cudaError_t nchw_to_nhwc_launch(const void* in, int in_fp32, __half* out, int C, int H, int W,
                                cudaStream_t s);
cudaError_t nhwc_to_nchw_launch(const __half* in, void* out, int out_fp32, int C, int H, int W,
                                cudaStream_t s);

}  // namespace ah
