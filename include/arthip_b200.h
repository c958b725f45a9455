/* arthip_b200 — C ABI of the B200-native fp16 conv-chain engine.
 *
 * All functions are plain C: pointers, sizes and ints only. Return codes follow the
 * reference's engine driver (tests/correctness/harness/engine_harness.cc:12-15):
 *   0 = ok, 1 = build / shape / argument failure, 2 = run failure.
 * Error text is copied (NUL-terminated, truncated) into the caller's `err` buffer.
 * Host IO buffers are NCHW plane-major in the model's IO dtype (fp16, or fp32 for
 * models with fp32 boundary Casts), exactly like vship::HipEngine::Run
 * (src/vapoursynth/hip_engine.h:100-105).
 */
#ifndef ARTHIP_B200_H
#define ARTHIP_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------------
 * Reference engine-driver ABI (drop-in for tests/correctness/harness/engine_harness.cc)
 * ---------------------------------------------------------------------------- */

/* Replaces engine_device_count (engine_harness.cc:56-63). */
int engine_device_count(int* count);

/* Replaces engine_probe (engine_harness.cc:65-94): build `model_path` on `device`,
 * report IO dtypes, the first conv's input channels / last conv's output channels and
 * the NCHW output shape for input [N, C, H, W]. */
int engine_probe(const char* model_path, int N, int H, int W, int C, int device, char* err, int errlen,
                 int* in_fp32, int* out_fp32, int* cin, int* cout, int64_t* out_shape, int* out_rank);

/* Replaces engine_run (engine_harness.cc:96-145): one frame through a fresh engine. */
int engine_run(const char* model_path, int N, int H, int W, int C, int device, const void* input,
               size_t input_bytes, void* out, size_t cap, size_t* out_bytes, int* out_fp32, int64_t* out_shape,
               int* out_rank, char* err, int errlen);

/* Replaces engine_alloc_failure_then_run (engine_harness.cc:151-210): an oversized frame
 * must fail with the allocation error and the same engine must then run a 16x16 frame. */
int engine_alloc_failure_then_run(const char* model_path, int N, int bigH, int bigW, int C, int device,
                                  const void* recovery_input, size_t recovery_input_bytes, void* out, size_t cap,
                                  size_t* out_bytes, int* out_fp32, int64_t* out_shape, int* out_rank,
                                  char* failerr, int failerrlen, char* runerr, int runerrlen);

/* ------------------------------------------------------------------------------
 * Persistent engine handle. Replaces the vship::HipEngine C++ object the VapourSynth
 * plugin holds per stream (src/vapoursynth/vs_hip.cpp:517-527, hip_engine.h:88-131) and
 * the hip::HipGraph the ORT EP compiles per partition (src/onnxruntime-hip/hip_graph.h:91-167).
 * ---------------------------------------------------------------------------- */
typedef struct ah_engine ah_engine;

/* HipEngine(int device_id) + Build(ModelProto) from a file or serialized bytes. */
int ah_engine_create_from_file(const char* model_path, int device, ah_engine** out, char* err, int errlen);
int ah_engine_create_from_bytes(const void* model, size_t model_bytes, int device, ah_engine** out, char* err,
                                int errlen);
void ah_engine_destroy(ah_engine* e);

/* InputIsFp32 / OutputIsFp32 / InputChannels / OutputChannels (hip_engine.h:118-131). */
int ah_engine_info(ah_engine* e, int* in_fp32, int* out_fp32, int* cin, int* cout);

/* GetOutputShape (hip_engine.h:96-98): NCHW in, NCHW out (4 values). */
int ah_engine_output_shape(ah_engine* e, int N, int C, int H, int W, int64_t* out_shape4);

/* Run (hip_engine.h:104-105): host NCHW input/output, synchronous, thread-safe.
 * Pinned (page-locked) host buffers are transferred directly; pageable ones through the
 * engine's pinned staging. */
int ah_engine_run(ah_engine* e, int N, int C, int H, int W, const void* input, size_t input_bytes, void* output,
                  size_t output_cap, char* err, int errlen);

/* Device-resident frames: build the plan for [N,C,H,W] and return the engine's device
 * boundary buffers (NCHW, model IO dtype; valid until the next shape change). */
int ah_engine_prepare(ah_engine* e, int N, int C, int H, int W, void** in_dev, void** out_dev, size_t* in_bytes,
                      size_t* out_bytes, char* err, int errlen);
/* Enqueue one frame (input buffer -> output buffer) on the engine's stream; asynchronous.
 * Replays a CUDA graph captured per resolution. */
int ah_engine_enqueue(ah_engine* e, char* err, int errlen);
int ah_engine_synchronize(ah_engine* e, char* err, int errlen);
/* Conv algorithm of the engine's 64 -> 64 layers (no counterpart setting in the reference,
 * which always runs Winograd): 0 = direct implicit GEMM on tcgen05 (default; exact fp16
 * products), 1 = Winograd F(2x2,3x3) on tcgen05 with fp16 transformed operands, the
 * reference's own numerics (accurate on trained models, outside a 4e-3 bar on deep
 * random-weight chains). The environment variable ARTHIP_CONV_ALGO=winograd selects 1 at
 * engine creation. Drops the current plan; returns 1 for another value. */
int ah_engine_set_conv_algo(ah_engine* e, int algo, char* err, int errlen);
/* Launch ops [begin, end) of the prepared plan directly on the engine stream, one kernel
 * each, no CUDA graph; asynchronous. For callers that put their own work between ops: the
 * per-layer 1-row halo exchange of a frame split into row strips across GPUs (the
 * reference has no split and rejects tiling, src/vapoursynth/vs_hip.cpp:466-494). */
int ah_engine_enqueue_ops(ah_engine* e, int begin, int end, char* err, int errlen);
/* Output buffer of op i of the prepared plan: device pointer, rows and bytes per row of its
 * NHWC fp16 layout (W x channels x 2), and boundary = 1 when it writes the model output
 * buffer (NCHW, IO dtype) instead. Returns 1 for a bad index or an unprepared engine. */
int ah_engine_op_output(ah_engine* e, int i, void** ptr, int* rows, size_t* row_bytes, int* boundary);
/* The engine's CUDA stream (cudaStream_t) for ordering caller copies with frames. */
void* ah_engine_stream(ah_engine* e);

/* Per-op timing over up to max_frames enqueued frames (CUDA events on the engine
 * stream); read returns per-op summed ms (n_ops entries) and the first-to-last span. */
int ah_engine_timing_start(ah_engine* e, int max_frames, char* err, int errlen);
int ah_engine_timing_read(ah_engine* e, double* op_ms, int n_ops, double* span_ms, int* frames, char* err,
                          int errlen);
/* Device op list of the prepared plan: kernel family, label, algorithmic FLOPs and bytes. */
int ah_engine_num_ops(ah_engine* e);
int ah_engine_op_info(ah_engine* e, int i, char* kind, int kindlen, char* label, int labellen, double* flops,
                      double* bytes);
/* Fused op list (one line per op), for inspection. */
int ah_engine_describe(ah_engine* e, char* buf, int len);

/* Parse + fuse a model without touching any GPU (fusion decisions / rejections). */
int ah_model_inspect(const char* model_path, char* buf, int len, int* in_fp32, int* out_fp32, int* cin,
                     int* cout, char* err, int errlen);

/* ------------------------------------------------------------------------------
 * ONNX Runtime execution-provider partition rules (the provider "HIPExecutionProvider",
 * src/onnxruntime-hip/hip_execution_provider.{h,cc}). The ORT-facing shim hands the
 * serialized model to these calls and maps the results onto ComputeCapability /
 * NodeComputeInfo; nothing here needs ORT headers. Nodes are identified by their position
 * in graph.node (ONNX node order is topological).
 * ---------------------------------------------------------------------------- */
typedef struct ah_ep_capability ah_ep_capability;

/* 1 when `device` exists and is an sm_100 GPU (the provider's context initializes),
 * else 0. HipExecutionProvider's constructor context check (hip_execution_provider.cc:164-175). */
int ah_ep_device_usable(int device);
/* IsNodeSupported (hip_execution_provider.cc:22-161) for node `node_index`, plus Relu:
 * 1 supported, 0 not, -1 malformed model. */
int ah_ep_node_supported(const void* model, size_t model_bytes, int node_index);
/* GetCapability (hip_execution_provider.cc:180-335): the maximal runs of supported nodes
 * that have exactly one activation input and one output. context_ok = 0 claims nothing,
 * as the reference does without a usable device. */
int ah_ep_get_capability(const void* model, size_t model_bytes, int context_ok, ah_ep_capability** out, char* err,
                         int errlen);
int ah_ep_region_count(const ah_ep_capability* c);
/* Node positions of region `region` (writes up to cap; returns the count, -1 bad index). */
int ah_ep_region_nodes(const ah_ep_capability* c, int region, int* nodes, int cap);
/* The region's MetaDef values: kind 0 = activation inputs, 1 = initializer inputs,
 * 2 = outputs. Count, then the j-th name. */
int ah_ep_region_value_count(const ah_ep_capability* c, int region, int kind);
int ah_ep_region_value(const ah_ep_capability* c, int region, int kind, int j, char* buf, int len);
/* MetaDef name "HipKernel_graph_<k>". */
int ah_ep_region_name(const ah_ep_capability* c, int region, char* buf, int len);
/* The fused op list the region compiles to, without a GPU (for inspection and tests). */
int ah_ep_region_inspect(const ah_ep_capability* c, int region, char* buf, int len, char* err, int errlen);
/* Compile (hip_execution_provider.cc:337-406): build an engine for the region on `device`;
 * run it with ah_engine_run (host NCHW IO in the region's IO dtype). Errors are prefixed
 * "HIP EP: ". */
int ah_ep_compile_region(const ah_ep_capability* c, int region, int device, ah_engine** out, char* err, int errlen);
void ah_ep_capability_destroy(ah_ep_capability* c);

/* ------------------------------------------------------------------------------
 * Single fused conv layer (3x3, stride 1, pad 1) on device NHWC fp16 tensors:
 * out = [add2 +] [add1 +] act(conv(in, w) + bias). Replaces one winograd_conv /
 * direct_conv dispatch (src/common/hip_kernels.h:143-483) as the engine issues it.
 * ---------------------------------------------------------------------------- */
typedef struct ah_conv ah_conv;

/* w_oihw_f16: [M][C][3][3] fp16 bit patterns (host); bias: M floats or NULL;
 * act: 0 none, 1 ReLU, 2 SiLU. */
int ah_conv3x3_create(int device, int C, int M, const uint16_t* w_oihw_f16, const float* bias, int act,
                      ah_conv** out, char* err, int errlen);
/* Enqueue on `stream` (cudaStream_t, NULL = legacy default). add1/add2 may be NULL; the
 * result is ((conv + add1) + add2), each sum rounded to fp16. out_nhwc may be the same
 * buffer as the last residual operand (an in-place residual update): the tensor-core
 * kernel then leaves that addition to reduce-add tile stores in L2, with the same result
 * bit for bit. It must not overlap in_nhwc. */
int ah_conv3x3_run(ah_conv* c, const void* in_nhwc, int H, int W, const void* add1, const void* add2,
                   void* out_nhwc, void* stream, char* err, int errlen);
/* The same layer on a chosen kernel (C = 64, M = 64 for algo 1 and 2; else return 1):
 * algo 0 = the default selection (as ah_conv3x3_create);
 * algo 1 = Winograd F(2x2,3x3) on tcgen05 with the reference's numerics (winograd_conv,
 *          src/common/hip_kernels.h:143-396; U = G g G^T rounded to fp16,
 *          src/vapoursynth/hip_engine.cc:972-1009), less exact than the direct form;
 * algo 2 = the direct vertical-window conv on two SMs per MMA (tcgen05 cta_group::2).
 * Run with ah_conv3x3_run. */
int ah_conv3x3_create_algo(int device, int C, int M, const uint16_t* w_oihw_f16, const float* bias, int act, int algo,
                           ah_conv** out, char* err, int errlen);
/* 0 = tcgen05 direct implicit GEMM, 1 = CUDA-core kernel, 2 = tcgen05 Winograd,
 * 3 = tcgen05 direct on two SMs. */
int ah_conv3x3_kind(ah_conv* c);
/* Reads and clears the device error word the tensor-core kernel writes on a timed-out
 * pipeline wait (0 = none). Synchronises the device. */
int ah_conv3x3_status(ah_conv* c, uint32_t* status);
void ah_conv3x3_destroy(ah_conv* c);

/* Allocation-free single conv layer (no counterpart in the reference; an addition of this
 * library). For callers that may not allocate GPU memory while they run a layer, such as
 * plugin hosts that give a plugin device buffers from their own pool and forbid cudaMalloc
 * inside it. Same arguments and result as ah_conv3x3_create + ah_conv3x3_run + status,
 * on the tensor-core kernel only (C % 16 == 0, C <= 128, M <= 256; anything else is rejected
 * with return 1 and a message). Calls no cudaMalloc / cudaFree: the packed weights, bias
 * and error word live in a fixed 591,104-byte __device__ array that every GPU that loads the
 * library keeps until exit. All calls on a device share that device's array, so calls on one
 * device are serialised on the host and each returns after its kernel has finished (work
 * overlapping on the GPU would race on the array); calls on different devices may run
 * concurrently. `stream` must belong to `device` (else return 1); the caller's current
 * device is restored on return. Each call looks up the array's device address with
 * cudaGetSymbolAddress, which allocates nothing; make the first call on a device before
 * any stream capture on it. Returns 0, 1 (bad arguments / unsupported) or 2 (CUDA error or
 * a timed-out pipeline wait). */
int ah_conv3x3_run_noalloc(int device, int C, int M, const uint16_t* w_oihw_f16, const float* bias, int act,
                           const void* in_nhwc, int H, int W, const void* add1, const void* add2,
                           void* out_nhwc, void* stream, char* err, int errlen);

/* Test-only failure-path hook (no counterpart in the reference). For tensor-core conv launches made after the call, in this process:
 * every pipeline wait is bounded by wait_limit_ms (1..4000) instead of 4 s, and every CTA
 * arms the slot of its input row `stall_row` (counted from the CTA's first row) without
 * loading it, so the kernel must report a timed-out wait through its status word without
 * faulting. Any other arguments (e.g. 0, -1) turn it off, which is the default. */
void ah_test_set_conv_fault_hook(int wait_limit_ms, int stall_row);

/* ------------------------------------------------------------------------------
 * VapourSynth filter hip.Model and its loading path (src/vapoursynth/vs_hip.cpp,
 * onnx_utils.cpp, convert_float_to_float16.cpp) as plain C: a plugin shim built against
 * VapourSynth4.h registers "Model" and maps VSMap arguments and VSFrame planes onto these.
 * Errors of the filter calls are prefixed "hip.Model: ".
 * ---------------------------------------------------------------------------- */

/* fp32 -> fp16 model conversion at load time (convert_float_to_float16.cpp:294-611):
 * fp32 initializers to fp16 with the converter's flush-to-zero rounding
 * (convert_float_to_float16.cpp:165-186), fp32 graph IO to fp16 unless cast_input /
 * cast_output keep it fp32 behind inserted boundary Casts, op types in the comma-separated
 * op_block_list (may be NULL) kept fp32 with Casts around them. Writes the serialized model
 * to `out` (out == NULL: only *out_bytes, the size); returns 1 on a parse error or a short
 * buffer. */
int ah_convert_float_to_float16(const void* model, size_t model_bytes, int force_fp16_initializers,
                                const char* op_block_list, int cast_input, int cast_output, void* out, size_t cap,
                                size_t* out_bytes, char* err, int errlen);
/* loadONNX (onnx_utils.cpp:29-128): the model from bytes (or, with model == NULL, from
 * `path`), one rank-4 input and one rank-4 output required; fixes the input to [1, C,
 * tile_h, tile_w] and the output batch to 1. Same output convention as above. */
int ah_load_onnx(const void* model, size_t model_bytes, const char* path, int64_t tile_w, int64_t tile_h, void* out,
                 size_t cap, size_t* out_bytes, char* err, int errlen);

/* A clip or frame format, in VapourSynth's terms (VSColorFamily: 0 undefined, 1 gray,
 * 2 RGB, 3 YUV; VSSampleType: 0 integer, 1 float). width / height are the luma plane's. */
typedef struct {
  int color_family;
  int sample_type;
  int bits_per_sample;
  int subsampling_w, subsampling_h;
  int num_planes;
  int width, height;
} ah_vs_format;

/* hip.Model's optional arguments (vs_hip.cpp:626-633). overlap / tilesize: number of
 * values given (0 = absent) and the values. fp16 defaults to 1 when fp16_set is 0.
 * flexible_output_prop: NULL or "" when absent. */
typedef struct {
  int device_id;
  int num_streams;
  int fp16_set;
  int64_t fp16;
  int overlap_n;
  int64_t overlap[2];
  int tilesize_n;
  int64_t tilesize[2];
  const char* flexible_output_prop;
} ah_vs_args;

typedef struct ah_vs_model ah_vs_model;

/* hipCreate (vs_hip.cpp:337-591): validates the clip (gray / YUV / RGB, 8/16-bit integer or
 * fp16/fp32, no subsampling) and the tiling arguments, loads the model from bytes (or from
 * network_path when model is NULL), converts it to fp16 when fp16 (boundary Casts kept for
 * fp32 clips), builds num_streams engines on device_id and checks the clip's plane count
 * against the model's input channels. */
int ah_vs_model_create(const ah_vs_format* clip, const void* model, size_t model_bytes, const char* network_path,
                       const ah_vs_args* args, ah_vs_model** out, char* err, int errlen);
/* The output clip format (gray, or RGB for a 3-channel output without the flexible
 * protocol; fp32, fp16 or 16-bit integer; the model's scale applied to width / height) and
 * the number of output channels (the flexible protocol's num_planes). */
int ah_vs_model_output(const ah_vs_model* m, ah_vs_format* out_format, int* num_output_channels);
/* hipGetFrame (vs_hip.cpp:77-321): one frame. src_planes / src_strides: the frame's planes
 * (bytes per row); the next engine of the pool (round-robin) runs it; output channel c is
 * written to dst_planes[c] for c < n_dst_planes. Thread-safe; returns 0, 1 (format) or 2
 * (run failure). */
int ah_vs_model_get_frame(ah_vs_model* m, const ah_vs_format* frame_format, const void* const* src_planes,
                          const ptrdiff_t* src_strides, void* const* dst_planes, const ptrdiff_t* dst_strides,
                          int n_dst_planes, char* err, int errlen);
void ah_vs_model_destroy(ah_vs_model* m);
/* hip.DeviceProperties (vs_hip.cpp:602-614): name, PCI device id, SM clock (kHz), global
 * memory (bytes). Returns 1 for a bad device. */
int ah_device_properties(int device, char* name, int namelen, int64_t* pci_device_id, int64_t* clock_rate_khz,
                         int64_t* global_memory);

/* ------------------------------------------------------------------------------
 * Host fp16 conversions used at load time (no GPU).
 * RNE: hip_engine.cc:1190-1232 (FloatToHalfBitsRNE). FTZ: convert_float_to_float16.cpp:165-186.
 * ---------------------------------------------------------------------------- */
void ah_float_to_half_rne(const float* in, uint16_t* out, size_t n);
void ah_float_to_half_ftz(const float* in, uint16_t* out, size_t n);
void ah_half_to_float(const uint16_t* in, float* out, size_t n);

const char* ah_version(void);

#ifdef __cplusplus
}
#endif

#endif /* ARTHIP_B200_H */
