// Conv-chain inference engine: ONNX graph -> fused op list -> per-resolution device plan
// (buffers, packed weights, kernel plans, CUDA graph) -> frames.
//
// This is the single engine core behind both front ends of the reference (the ONNX
// Runtime execution provider's compiled graph, src/onnxruntime-hip/hip_graph.{h,cc}, and
// the VapourSynth plugin's standalone engine, src/vapoursynth/hip_engine.{h,cc}). The
// public contract follows vship::HipEngine (hip_engine.h:88-131): Build() parses and fuses
// the model, GetOutputShape() propagates an NCHW shape, Run() takes and returns host NCHW
// buffers in the model's IO dtype, is synchronous, returns false with a message on
// failure, and leaves the engine usable afterwards.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <limits>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "kernels/kernels.h"
#include "onnx_wire.h"

namespace ah {

enum class OpType { Conv, Sigmoid, Mul, Add, Clip, Relu, DepthToSpace };

const char* OpTypeName(OpType t);

struct OpSpec {
  OpType type = OpType::Conv;
  std::string in0;
  std::string in1;  // binary operand, or the Conv weight initializer
  std::string out;
  std::string bias;                 // Conv bias initializer (may be empty)
  int act = kActNone;               // fused epilogue activation (Conv)
  std::vector<std::string> adds;    // fused residual operands, applied in order (Conv, <= 2)
  float clip_min = -std::numeric_limits<float>::infinity();
  float clip_max = std::numeric_limits<float>::infinity();
  bool fuse_clip = false;           // DepthToSpace (or a Conv with fuse_dts): clip folded in
  int blocksize = 1;                // DepthToSpace block size
  bool fuse_dts = false;            // Conv writes DepthToSpace(DCR) of its result
};

struct WeightSpec {
  std::vector<uint8_t> data;
  std::vector<int64_t> shape;
  int dtype = 0;
};

class Engine {
 public:
  explicit Engine(int device_id = 0);
  ~Engine();
  Engine(const Engine&) = delete;
  Engine& operator=(const Engine&) = delete;

  // Parse + fuse the model, then select the device and create the stream.
  bool Build(const onnx::Model& model, std::string& error);
  // Parse + fuse only (no CUDA calls): used to inspect fusion decisions on any host.
  bool BuildHostOnly(const onnx::Model& model, std::string& error);

  bool GetOutputShape(const std::vector<int64_t>& in_nchw, std::vector<int64_t>& out_nchw) const;

  // Host NCHW buffers in the model IO dtype; synchronous.
  bool Run(const void* input, const std::vector<int64_t>& in_nchw, void* output, std::string& error);

  // Device-resident path: build the plan for `in_nchw` and expose the device boundary
  // buffers (NCHW, model IO dtype). Enqueue() runs one frame on the engine stream from
  // the input buffer to the output buffer without synchronising.
  bool Prepare(const std::vector<int64_t>& in_nchw, void** in_dev, void** out_dev, size_t* in_bytes,
               size_t* out_bytes, std::string& error);
  bool Enqueue(std::string& error);
  // Launch ops [begin, end) of the prepared plan directly on the engine stream (no CUDA
  // graph), so a caller can put its own work between ops (the per-layer halo exchange of
  // a row-strip split).
  bool EnqueueOps(int begin, int end, std::string& error);
  // Output buffer of op i: device pointer, rows (the op's H) and bytes per row (W x
  // channels fp16, NHWC), and whether it is the boundary output (NCHW, IO dtype: then
  // rows / row_bytes describe the NHWC shape of the op, not the boundary layout).
  bool OpOutput(int i, void** ptr, int* rows, size_t* row_bytes, bool* boundary) const;
  bool Synchronize(std::string& error);
  cudaStream_t stream() const { return stream_; }
  // Conv algorithm for 64 -> 64 layers: 0 = direct implicit GEMM (default, exact fp16
  // products), 1 = Winograd F(2x2,3x3) with fp16 transformed operands (the reference's
  // numerics). Also set by ARTHIP_CONV_ALGO=winograd at construction. Drops the current plan.
  bool SetConvAlgo(int algo, std::string& error);

  // Per-op timing over many frames (CUDA events on the engine stream, no host sync per
  // frame): TimingStart reserves events for up to max_frames; Enqueue then launches ops
  // directly with events around each; TimingRead returns the per-op summed milliseconds
  // and the span from the first frame's start to the last frame's end.
  bool TimingStart(int max_frames, std::string& error);
  bool TimingRead(std::vector<double>* op_ms, double* span_ms, int* frames, std::string& error);

  struct OpInfo {
    std::string kind;     // kernel family: "conv_tc", "conv_simt", "unary", "binary", "dts", "io"
    std::string label;    // op description
    double flops = 0.0;   // algorithmic FLOPs (direct conv count)
    double bytes = 0.0;   // algorithmic HBM bytes (each operand read once, output written once)
  };
  std::vector<OpInfo> DeviceOps() const;

  bool InputIsFp32() const { return input_is_fp32_; }
  bool OutputIsFp32() const { return output_is_fp32_; }
  int InputChannels() const;
  int OutputChannels() const;
  std::string Describe() const;  // fused op list, one line per op
  int device() const { return device_id_; }

 private:
  struct DevOp {
    OpType type = OpType::Conv;
    int kind = 0;  // 0 conv_tc, 1 conv_simt, 2 unary, 3 binary, 4 dts, 5 nchw->nhwc, 6 nhwc->nchw, 7 conv_wino
    int in_buf = -1, in1_buf = -1, add_buf[2] = {-1, -1}, out_buf = -1;
    bool out_boundary = false;  // writes the boundary output buffer
    bool in_boundary = false;   // reads the boundary input buffer
    int H = 0, W = 0, C = 0, M = 0;
    int act = kActNone;
    int widx = -1;  // conv weights index
    ConvTcPlan tc;
    WinoPlan wp;
    SimtOut sout;
    size_t numel = 0;
    int subop = 0;
    float lo = 0.f, hi = 0.f;
    OpInfo info;
  };
  struct ConvWeights {
    bool tc = false;
    bool wino = false;
    ConvTcWeights tcw;
    SimtConvWeights sw;
    WinoWeights ww;
  };

  bool Parse(const onnx::Model& model, std::string& error);
  bool PropagateShapes(const std::vector<int64_t>& in_nchw,
                       std::unordered_map<std::string, std::vector<int64_t>>& shapes) const;
  bool EnsureBuilt(const std::vector<int64_t>& in_nchw, std::string& error);
  bool UploadWeights(std::string& error);
  void FreeWeights();
  bool LaunchFrame(bool with_events, std::string& error);
  cudaError_t LaunchOp(size_t i, cudaStream_t s);
  bool CheckStatus(std::string& error);
  void DestroyShapeState();
  void DestroyAll();
  bool SetDevice(std::string& error) const;
  void* BufPtr(int idx) const;

  int device_id_ = 0;
  cudaStream_t stream_ = nullptr;
  bool device_ready_ = false;
  int conv_algo_ = 0;
  int num_sms_ = 148;

  std::string input_name_, output_name_;
  std::vector<OpSpec> ops_;
  std::unordered_map<std::string, WeightSpec> weights_;
  bool input_is_fp32_ = false, output_is_fp32_ = false;

  // weights uploaded once per model (index = position in ops_ among convs)
  std::vector<ConvWeights> conv_weights_;
  std::vector<int> conv_widx_;  // ops_ index -> conv_weights_ index
  bool weights_uploaded_ = false;

  // per-shape state
  bool built_ = false;
  std::vector<int64_t> built_shape_;
  std::vector<void*> bufs_;
  std::vector<size_t> buf_bytes_;
  std::unordered_map<std::string, int> tensor_buf_;
  std::vector<DevOp> dev_ops_;
  void* in_boundary_ = nullptr;   // device, NCHW in the model input dtype (owned unless aliased)
  void* out_boundary_ = nullptr;  // device, NCHW in the model output dtype
  bool in_alias_ = false, out_alias_ = false;
  size_t in_bytes_ = 0, out_bytes_ = 0;
  void* in_staging_ = nullptr;    // pinned host
  void* out_staging_ = nullptr;   // pinned host
  uint32_t* status_ = nullptr;    // device error word written by kernels
  cudaGraphExec_t graph_exec_ = nullptr;

  // timing
  std::vector<cudaEvent_t> tevents_;
  int t_max_frames_ = 0, t_frames_ = 0;

  // diagnostics (env knobs, reference names)
  bool prof_ = false, trace_ = false, poison_ = false, sync_each_ = false, no_graph_ = false;
  uint64_t frame_no_ = 0;
  std::vector<cudaEvent_t> prof_events_;

  mutable std::mutex mutex_;
};

}  // namespace ah
