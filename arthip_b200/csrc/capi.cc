// extern "C" boundary of the engine (declarations and reference mapping in
// include/arthip_b200.h).
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "../../include/arthip_b200.h"
#include "engine.h"
#include "ep_partition.h"
#include "fp16_host.h"
#include "kernels/kernels.h"

namespace {

constexpr int kMaxRank = 8;

void CopyOut(const std::string& s, char* dst, int len) {
  if (!dst || len <= 0) return;
  size_t n = s.size();
  if (n > static_cast<size_t>(len) - 1) n = static_cast<size_t>(len) - 1;
  std::memcpy(dst, s.data(), n);
  dst[n] = '\0';
}

void WriteShape(const std::vector<int64_t>& s, int64_t* out, int* rank) {
  if (rank) *rank = static_cast<int>(s.size());
  if (!out) return;
  for (size_t i = 0; i < s.size() && i < static_cast<size_t>(kMaxRank); ++i) out[i] = s[i];
}

size_t Elem(bool fp32) { return fp32 ? 4u : 2u; }

bool LoadAndBuild(const char* path, int device, ah::Engine* eng, std::string* err) {
  ah::onnx::Model m;
  if (!path || !ah::onnx::LoadModelFile(path, &m, err)) {
    if (err && err->empty()) *err = "failed to parse model file";
    return false;
  }
  return eng->Build(m, *err);
}

}  // namespace

struct ah_engine {
  std::unique_ptr<ah::Engine> eng;
};

struct ah_ep_capability {
  ah::onnx::Model model;
  std::vector<ah::ep::Region> regions;
};

struct ah_conv {
  int device = 0;
  int C = 0, M = 0, act = 0;
  bool tc = false;
  bool wino = false;
  bool pair = false;
  ah::ConvTcWeights tcw;
  ah::SimtConvWeights sw;
  ah::WinoWeights ww;
  ah::WinoPlan wplan;
  ah::PairWeights pw;
  ah::PairPlan pplan;
  ah::ConvTcPlan plan;
  const void* plan_in = nullptr;
  const void* plan_out = nullptr;
  int plan_H = 0, plan_W = 0;
  int num_sms = 148;
  uint32_t* status = nullptr;
};

extern "C" {

// ---------------------------------------------------------------------------
// Reference engine-driver ABI
// ---------------------------------------------------------------------------
int engine_device_count(int* count) {
  if (!count) return 1;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    (void)cudaGetLastError();
    return 1;
  }
  *count = n;
  return 0;
}

int engine_probe(const char* model_path, int N, int H, int W, int C, int device, char* err, int errlen,
                 int* in_fp32, int* out_fp32, int* cin, int* cout, int64_t* out_shape, int* out_rank) {
  ah::Engine eng(device);
  std::string e;
  if (!LoadAndBuild(model_path, device, &eng, &e)) {
    CopyOut(e, err, errlen);
    return 1;
  }
  if (in_fp32) *in_fp32 = eng.InputIsFp32();
  if (out_fp32) *out_fp32 = eng.OutputIsFp32();
  if (cin) *cin = eng.InputChannels();
  if (cout) *cout = eng.OutputChannels();
  std::vector<int64_t> shape;
  if (!eng.GetOutputShape({N, C, H, W}, shape)) {
    CopyOut("shape propagation failed", err, errlen);
    return 1;
  }
  WriteShape(shape, out_shape, out_rank);
  CopyOut("", err, errlen);
  return 0;
}

int engine_run(const char* model_path, int N, int H, int W, int C, int device, const void* input,
               size_t input_bytes, void* out, size_t cap, size_t* out_bytes, int* out_fp32, int64_t* out_shape,
               int* out_rank, char* err, int errlen) {
  ah::Engine eng(device);
  std::string e;
  if (!LoadAndBuild(model_path, device, &eng, &e)) {
    CopyOut(e, err, errlen);
    return 1;
  }
  std::vector<int64_t> in_shape{N, C, H, W}, shape;
  if (!eng.GetOutputShape(in_shape, shape) || shape.size() != 4) {
    CopyOut("shape propagation failed", err, errlen);
    return 1;
  }
  const bool o32 = eng.OutputIsFp32();
  const size_t need = static_cast<size_t>(shape[0] * shape[1] * shape[2] * shape[3]) * Elem(o32);
  if (need > cap) {
    CopyOut("output buffer too small", err, errlen);
    return 1;
  }
  const size_t expect = static_cast<size_t>(N) * C * H * W * Elem(eng.InputIsFp32());
  if (!input || input_bytes != expect) {
    CopyOut("input buffer size mismatch (expected " + std::to_string(expect) + " bytes, got " +
                std::to_string(input_bytes) + ")",
            err, errlen);
    return 1;
  }
  if (!eng.Run(input, in_shape, out, e)) {
    CopyOut(e, err, errlen);
    return 2;
  }
  if (out_bytes) *out_bytes = need;
  if (out_fp32) *out_fp32 = o32;
  WriteShape(shape, out_shape, out_rank);
  CopyOut("", err, errlen);
  return 0;
}

int engine_alloc_failure_then_run(const char* model_path, int N, int bigH, int bigW, int C, int device,
                                  const void* recovery_input, size_t recovery_input_bytes, void* out, size_t cap,
                                  size_t* out_bytes, int* out_fp32, int64_t* out_shape, int* out_rank,
                                  char* failerr, int failerrlen, char* runerr, int runerrlen) {
  ah::Engine eng(device);
  std::string e;
  if (!LoadAndBuild(model_path, device, &eng, &e)) {
    CopyOut("build failed: " + e, failerr, failerrlen);
    return 1;
  }
  char dummy[8] = {0};
  std::string first;
  if (eng.Run(dummy, {N, C, bigH, bigW}, dummy, first)) {
    CopyOut("expected the oversized run to fail but it succeeded", failerr, failerrlen);
    return 1;
  }
  CopyOut(first, failerr, failerrlen);
  const int rh = 16, rw = 16;
  std::vector<int64_t> in_shape{N, C, rh, rw}, shape;
  if (!eng.GetOutputShape(in_shape, shape) || shape.size() != 4) {
    CopyOut("recovery shape probe failed", runerr, runerrlen);
    return 2;
  }
  const bool o32 = eng.OutputIsFp32();
  const size_t need = static_cast<size_t>(shape[0] * shape[1] * shape[2] * shape[3]) * Elem(o32);
  if (need > cap) {
    CopyOut("recovery output buffer too small", runerr, runerrlen);
    return 2;
  }
  const size_t expect = static_cast<size_t>(N) * C * rh * rw * Elem(eng.InputIsFp32());
  if (!recovery_input || recovery_input_bytes != expect) {
    CopyOut("recovery input buffer size mismatch", runerr, runerrlen);
    return 2;
  }
  std::string second;
  if (!eng.Run(recovery_input, in_shape, out, second)) {
    CopyOut(second, runerr, runerrlen);
    return 2;
  }
  if (out_bytes) *out_bytes = need;
  if (out_fp32) *out_fp32 = o32;
  WriteShape(shape, out_shape, out_rank);
  CopyOut("", runerr, runerrlen);
  return 0;
}

// ---------------------------------------------------------------------------
// Engine handle
// ---------------------------------------------------------------------------
static int CreateCommon(ah::onnx::Model& m, int device, ah_engine** out, char* err, int errlen) {
  if (!out) {
    CopyOut("null output handle", err, errlen);
    return 1;
  }
  auto h = std::make_unique<ah_engine>();
  h->eng = std::make_unique<ah::Engine>(device);
  std::string e;
  if (!h->eng->Build(m, e)) {
    CopyOut(e, err, errlen);
    return 1;
  }
  *out = h.release();
  CopyOut("", err, errlen);
  return 0;
}

int ah_engine_create_from_file(const char* model_path, int device, ah_engine** out, char* err, int errlen) {
  ah::onnx::Model m;
  std::string e;
  if (!model_path || !ah::onnx::LoadModelFile(model_path, &m, &e)) {
    CopyOut(e.empty() ? "failed to parse model file" : e, err, errlen);
    return 1;
  }
  return CreateCommon(m, device, out, err, errlen);
}

int ah_engine_create_from_bytes(const void* model, size_t model_bytes, int device, ah_engine** out, char* err,
                                int errlen) {
  ah::onnx::Model m;
  std::string e;
  if (!model || !ah::onnx::ParseModel(static_cast<const uint8_t*>(model), model_bytes, &m, &e)) {
    CopyOut(e.empty() ? "failed to parse model bytes" : e, err, errlen);
    return 1;
  }
  return CreateCommon(m, device, out, err, errlen);
}

void ah_engine_destroy(ah_engine* e) { delete e; }

int ah_engine_info(ah_engine* e, int* in_fp32, int* out_fp32, int* cin, int* cout) {
  if (!e) return 1;
  if (in_fp32) *in_fp32 = e->eng->InputIsFp32();
  if (out_fp32) *out_fp32 = e->eng->OutputIsFp32();
  if (cin) *cin = e->eng->InputChannels();
  if (cout) *cout = e->eng->OutputChannels();
  return 0;
}

int ah_engine_output_shape(ah_engine* e, int N, int C, int H, int W, int64_t* out_shape4) {
  if (!e || !out_shape4) return 1;
  std::vector<int64_t> s;
  if (!e->eng->GetOutputShape({N, C, H, W}, s)) return 1;
  for (int i = 0; i < 4; ++i) out_shape4[i] = s[i];
  return 0;
}

int ah_engine_run(ah_engine* e, int N, int C, int H, int W, const void* input, size_t input_bytes, void* output,
                  size_t output_cap, char* err, int errlen) {
  if (!e) {
    CopyOut("null engine", err, errlen);
    return 1;
  }
  std::vector<int64_t> in{N, C, H, W}, s;
  if (!e->eng->GetOutputShape(in, s)) {
    CopyOut("shape propagation failed", err, errlen);
    return 1;
  }
  const size_t need = static_cast<size_t>(s[0] * s[1] * s[2] * s[3]) * Elem(e->eng->OutputIsFp32());
  const size_t expect = static_cast<size_t>(N) * C * H * W * Elem(e->eng->InputIsFp32());
  if (need > output_cap) {
    CopyOut("output buffer too small", err, errlen);
    return 1;
  }
  if (!input || input_bytes != expect) {
    CopyOut("input buffer size mismatch (expected " + std::to_string(expect) + " bytes, got " +
                std::to_string(input_bytes) + ")",
            err, errlen);
    return 1;
  }
  std::string msg;
  if (!e->eng->Run(input, in, output, msg)) {
    CopyOut(msg, err, errlen);
    return 2;
  }
  CopyOut("", err, errlen);
  return 0;
}

int ah_engine_prepare(ah_engine* e, int N, int C, int H, int W, void** in_dev, void** out_dev, size_t* in_bytes,
                      size_t* out_bytes, char* err, int errlen) {
  if (!e) return 1;
  std::string msg;
  if (!e->eng->Prepare({N, C, H, W}, in_dev, out_dev, in_bytes, out_bytes, msg)) {
    CopyOut(msg, err, errlen);
    return 1;
  }
  return 0;
}

int ah_engine_enqueue(ah_engine* e, char* err, int errlen) {
  if (!e) return 1;
  std::string msg;
  if (!e->eng->Enqueue(msg)) {
    CopyOut(msg, err, errlen);
    return 2;
  }
  return 0;
}

int ah_engine_synchronize(ah_engine* e, char* err, int errlen) {
  if (!e) return 1;
  std::string msg;
  if (!e->eng->Synchronize(msg)) {
    CopyOut(msg, err, errlen);
    return 2;
  }
  return 0;
}

int ah_engine_set_conv_algo(ah_engine* e, int algo, char* err, int errlen) {
  if (!e) return 1;
  std::string msg;
  if (!e->eng->SetConvAlgo(algo, msg)) {
    CopyOut(msg, err, errlen);
    return 1;
  }
  return 0;
}

int ah_engine_enqueue_ops(ah_engine* e, int begin, int end, char* err, int errlen) {
  if (!e) return 1;
  std::string msg;
  if (!e->eng->EnqueueOps(begin, end, msg)) {
    CopyOut(msg, err, errlen);
    return 2;
  }
  return 0;
}

int ah_engine_op_output(ah_engine* e, int i, void** ptr, int* rows, size_t* row_bytes, int* boundary) {
  if (!e || !ptr || !rows || !row_bytes || !boundary) return 1;
  bool b = false;
  if (!e->eng->OpOutput(i, ptr, rows, row_bytes, &b)) return 1;
  *boundary = b ? 1 : 0;
  return 0;
}

void* ah_engine_stream(ah_engine* e) { return e ? static_cast<void*>(e->eng->stream()) : nullptr; }

int ah_engine_timing_start(ah_engine* e, int max_frames, char* err, int errlen) {
  if (!e) return 1;
  std::string msg;
  if (!e->eng->TimingStart(max_frames, msg)) {
    CopyOut(msg, err, errlen);
    return 1;
  }
  return 0;
}

int ah_engine_timing_read(ah_engine* e, double* op_ms, int n_ops, double* span_ms, int* frames, char* err,
                          int errlen) {
  if (!e) return 1;
  std::vector<double> v;
  std::string msg;
  double span = 0;
  int f = 0;
  const bool ok = e->eng->TimingRead(&v, &span, &f, msg);
  if (op_ms)
    for (int i = 0; i < n_ops && i < static_cast<int>(v.size()); ++i) op_ms[i] = v[i];
  if (span_ms) *span_ms = span;
  if (frames) *frames = f;
  if (!ok) {
    CopyOut(msg, err, errlen);
    return 2;
  }
  return 0;
}

int ah_engine_num_ops(ah_engine* e) { return e ? static_cast<int>(e->eng->DeviceOps().size()) : -1; }

int ah_engine_op_info(ah_engine* e, int i, char* kind, int kindlen, char* label, int labellen, double* flops,
                      double* bytes) {
  if (!e) return 1;
  const auto ops = e->eng->DeviceOps();
  if (i < 0 || i >= static_cast<int>(ops.size())) return 1;
  CopyOut(ops[i].kind, kind, kindlen);
  CopyOut(ops[i].label, label, labellen);
  if (flops) *flops = ops[i].flops;
  if (bytes) *bytes = ops[i].bytes;
  return 0;
}

int ah_engine_describe(ah_engine* e, char* buf, int len) {
  if (!e) return 1;
  CopyOut(e->eng->Describe(), buf, len);
  return 0;
}

int ah_model_inspect(const char* model_path, char* buf, int len, int* in_fp32, int* out_fp32, int* cin, int* cout,
                     char* err, int errlen) {
  ah::onnx::Model m;
  std::string e;
  if (!model_path || !ah::onnx::LoadModelFile(model_path, &m, &e)) {
    CopyOut(e.empty() ? "failed to parse model file" : e, err, errlen);
    return 1;
  }
  ah::Engine eng(0);
  if (!eng.BuildHostOnly(m, e)) {
    CopyOut(e, err, errlen);
    return 1;
  }
  CopyOut(eng.Describe(), buf, len);
  if (in_fp32) *in_fp32 = eng.InputIsFp32();
  if (out_fp32) *out_fp32 = eng.OutputIsFp32();
  if (cin) *cin = eng.InputChannels();
  if (cout) *cout = eng.OutputChannels();
  CopyOut("", err, errlen);
  return 0;
}

// ---------------------------------------------------------------------------
// Single conv layer
// ---------------------------------------------------------------------------
int ah_conv3x3_create(int device, int C, int M, const uint16_t* w, const float* bias, int act, ah_conv** out,
                      char* err, int errlen) {
  if (!out || !w || C <= 0 || M <= 0 || C > 256 || M > 256) {
    CopyOut("invalid conv arguments", err, errlen);
    return 1;
  }
  cudaError_t ce = cudaSetDevice(device);
  if (ce != cudaSuccess) {
    CopyOut(std::string("cudaSetDevice(") + std::to_string(device) + ") failed: " + cudaGetErrorString(ce), err,
            errlen);
    (void)cudaGetLastError();
    return 1;
  }
  auto c = std::make_unique<ah_conv>();
  c->device = device;
  c->C = C;
  c->M = M;
  c->act = act;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) == cudaSuccess && sms > 0) c->num_sms = sms;
  c->tc = ah::conv_tc_supported(C, M, nullptr);
  ce = c->tc ? ah::conv_tc_upload(w, bias, C, M, &c->tcw) : ah::simt_conv_upload(w, bias, C, M, &c->sw);
  if (ce == cudaSuccess) ce = cudaMalloc(&c->status, sizeof(uint32_t));
  if (ce == cudaSuccess) ce = cudaMemset(c->status, 0, sizeof(uint32_t));
  if (ce != cudaSuccess) {
    CopyOut(std::string("conv weight upload failed: ") + cudaGetErrorString(ce), err, errlen);
    (void)cudaGetLastError();
    ah::conv_tc_free(&c->tcw);
    ah::simt_conv_free(&c->sw);
    if (c->status) cudaFree(c->status);
    return 1;
  }
  *out = c.release();
  return 0;
}

int ah_conv3x3_create_algo(int device, int C, int M, const uint16_t* w, const float* bias, int act, int algo,
                           ah_conv** out, char* err, int errlen) {
  if (algo == 0) return ah_conv3x3_create(device, C, M, w, bias, act, out, err, errlen);
  if (!out || !w || act < 0 || act > 2 || (algo != 1 && algo != 2)) {
    CopyOut("invalid conv arguments", err, errlen);
    return 1;
  }
  const bool ok = algo == 1 ? ah::wino_supported(C, M) : ah::pair_supported(C, M);
  if (!ok) {
    CopyOut(std::string(algo == 1 ? "Winograd" : "two-SM") + " conv supports C = 64, M = 64 (got C=" +
                std::to_string(C) + ", M=" + std::to_string(M) + ")",
            err, errlen);
    return 1;
  }
  cudaError_t ce = cudaSetDevice(device);
  if (ce != cudaSuccess) {
    CopyOut(std::string("cudaSetDevice(") + std::to_string(device) + ") failed: " + cudaGetErrorString(ce), err,
            errlen);
    (void)cudaGetLastError();
    return 1;
  }
  auto c = std::make_unique<ah_conv>();
  c->device = device;
  c->C = C;
  c->M = M;
  c->act = act;
  c->wino = algo == 1;
  c->pair = algo == 2;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) == cudaSuccess && sms > 0) c->num_sms = sms;
  ce = c->wino ? ah::wino_upload(w, bias, C, M, &c->ww) : ah::pair_upload(w, bias, C, M, &c->pw);
  if (ce == cudaSuccess) ce = cudaMalloc(&c->status, sizeof(uint32_t));
  if (ce == cudaSuccess) ce = cudaMemset(c->status, 0, sizeof(uint32_t));
  if (ce != cudaSuccess) {
    CopyOut(std::string("conv weight upload failed: ") + cudaGetErrorString(ce), err, errlen);
    (void)cudaGetLastError();
    ah::wino_free(&c->ww);
    ah::pair_free(&c->pw);
    if (c->status) cudaFree(c->status);
    return 1;
  }
  *out = c.release();
  return 0;
}

int ah_conv3x3_run(ah_conv* c, const void* in, int H, int W, const void* add1, const void* add2, void* out,
                   void* stream, char* err, int errlen) {
  if (!c || !in || !out || H <= 0 || W <= 0) {
    CopyOut("invalid conv run arguments", err, errlen);
    return 1;
  }
  cudaSetDevice(c->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (c->pair) {
    if (c->plan_in != in || c->plan_out != out || c->plan_H != H || c->plan_W != W) {
      std::string perr;
      if (!ah::pair_plan(&c->pw, static_cast<const __half*>(in), H, W, static_cast<__half*>(out), c->num_sms,
                         &c->pplan, &perr)) {
        CopyOut(perr, err, errlen);
        return 1;
      }
      c->plan_in = in;
      c->plan_out = out;
      c->plan_H = H;
      c->plan_W = W;
    }
    e = ah::pair_launch(c->pplan, static_cast<const __half*>(add1), static_cast<const __half*>(add2), c->act,
                        c->status, s);
  } else if (c->wino) {
    if (c->plan_in != in || c->plan_out != out || c->plan_H != H || c->plan_W != W) {
      std::string perr;
      if (!ah::wino_plan(&c->ww, static_cast<const __half*>(in), H, W, static_cast<__half*>(out), c->num_sms,
                         &c->wplan, &perr)) {
        CopyOut(perr, err, errlen);
        return 1;
      }
      c->plan_in = in;
      c->plan_out = out;
      c->plan_H = H;
      c->plan_W = W;
    }
    e = ah::wino_launch(c->wplan, static_cast<const __half*>(add1), static_cast<const __half*>(add2), c->act,
                        c->status, s);
  } else if (c->tc) {
    if (c->plan_in != in || c->plan_out != out || c->plan_H != H || c->plan_W != W) {
      std::string perr;
      ah::ConvTcOut to;
      to.ptr = out;
      to.mode = (c->M % 16 == 0) ? 0 : 1;  // NHWC via TMA stores, or per-element NHWC stores
      if (!ah::conv_tc_plan(&c->tcw, static_cast<const __half*>(in), H, W, to, c->num_sms, &c->plan, &perr)) {
        CopyOut(perr, err, errlen);
        return 1;
      }
      c->plan_in = in;
      c->plan_out = out;
      c->plan_H = H;
      c->plan_W = W;
    }
    e = ah::conv_tc_launch(c->plan, static_cast<const __half*>(add1), static_cast<const __half*>(add2), c->act,
                           c->status, s);
  } else {
    ah::SimtOut so;
    so.ptr = out;
    e = ah::simt_conv_launch(c->sw, static_cast<const __half*>(in), H, W, static_cast<const __half*>(add1),
                             static_cast<const __half*>(add2), c->act, so, s);
  }
  if (e != cudaSuccess) {
    CopyOut(std::string("conv launch failed: ") + cudaGetErrorString(e), err, errlen);
    (void)cudaGetLastError();
    return 2;
  }
  return 0;
}

int ah_conv3x3_kind(ah_conv* c) { return c ? (c->pair ? 3 : (c->wino ? 2 : (c->tc ? 0 : 1))) : -1; }

int ah_conv3x3_status(ah_conv* c, uint32_t* status) {
  if (!c || !status) return 1;
  cudaSetDevice(c->device);
  if (cudaDeviceSynchronize() != cudaSuccess) return 2;
  if (cudaMemcpy(status, c->status, sizeof(uint32_t), cudaMemcpyDeviceToHost) != cudaSuccess) return 2;
  cudaMemset(c->status, 0, sizeof(uint32_t));
  return 0;
}

void ah_conv3x3_destroy(ah_conv* c) {
  if (!c) return;
  cudaSetDevice(c->device);
  ah::conv_tc_free(&c->tcw);
  ah::simt_conv_free(&c->sw);
  ah::wino_free(&c->ww);
  ah::pair_free(&c->pw);
  if (c->status) cudaFree(c->status);
  delete c;
}

void ah_test_set_conv_fault_hook(int wait_limit_ms, int stall_row) {
  ah::conv_tc_set_test_hook(wait_limit_ms, stall_row);
}

// ---------------------------------------------------------------------------
// ONNX Runtime execution-provider partition rules
// ---------------------------------------------------------------------------
int ah_ep_device_usable(int device) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
    (void)cudaGetLastError();
    return 0;
  }
  cudaDeviceProp p;
  if (cudaGetDeviceProperties(&p, device) != cudaSuccess) {
    (void)cudaGetLastError();
    return 0;
  }
  return p.major == 10 ? 1 : 0;  // the kernels are built for sm_100a only
}

int ah_ep_node_supported(const void* model, size_t model_bytes, int node_index) {
  ah::onnx::Model m;
  std::string e;
  if (!model || !ah::onnx::ParseModel(static_cast<const uint8_t*>(model), model_bytes, &m, &e)) return -1;
  return ah::ep::IsNodeSupported(m.graph, node_index, ah::ep::InferElemTypes(m.graph)) ? 1 : 0;
}

int ah_ep_get_capability(const void* model, size_t model_bytes, int context_ok, ah_ep_capability** out, char* err,
                         int errlen) {
  if (!model || !out) {
    CopyOut("invalid capability arguments", err, errlen);
    return 1;
  }
  auto c = std::make_unique<ah_ep_capability>();
  std::string e;
  if (!ah::onnx::ParseModel(static_cast<const uint8_t*>(model), model_bytes, &c->model, &e)) {
    CopyOut("HIP EP: " + (e.empty() ? std::string("malformed model") : e), err, errlen);
    return 1;
  }
  c->regions = ah::ep::GetCapability(c->model, context_ok != 0);
  *out = c.release();
  return 0;
}

int ah_ep_region_count(const ah_ep_capability* c) { return c ? static_cast<int>(c->regions.size()) : -1; }

static const ah::ep::Region* EpRegion(const ah_ep_capability* c, int i) {
  if (!c || i < 0 || i >= static_cast<int>(c->regions.size())) return nullptr;
  return &c->regions[i];
}

int ah_ep_region_nodes(const ah_ep_capability* c, int region, int* nodes, int cap) {
  const auto* r = EpRegion(c, region);
  if (!r) return -1;
  for (int i = 0; i < static_cast<int>(r->nodes.size()) && nodes && i < cap; ++i) nodes[i] = r->nodes[i];
  return static_cast<int>(r->nodes.size());
}

static const std::vector<std::string>* EpValues(const ah::ep::Region* r, int kind) {
  if (!r) return nullptr;
  if (kind == 0) return &r->activations;
  if (kind == 1) return &r->constants;
  if (kind == 2) return &r->outputs;
  return nullptr;
}

int ah_ep_region_value_count(const ah_ep_capability* c, int region, int kind) {
  const auto* v = EpValues(EpRegion(c, region), kind);
  return v ? static_cast<int>(v->size()) : -1;
}

int ah_ep_region_value(const ah_ep_capability* c, int region, int kind, int j, char* buf, int len) {
  const auto* v = EpValues(EpRegion(c, region), kind);
  if (!v || j < 0 || j >= static_cast<int>(v->size())) return 1;
  CopyOut((*v)[j], buf, len);
  return 0;
}

int ah_ep_region_name(const ah_ep_capability* c, int region, char* buf, int len) {
  const auto* r = EpRegion(c, region);
  if (!r) return 1;
  CopyOut(r->name, buf, len);
  return 0;
}

int ah_ep_region_inspect(const ah_ep_capability* c, int region, char* buf, int len, char* err, int errlen) {
  const auto* r = EpRegion(c, region);
  if (!r) {
    CopyOut("no such region", err, errlen);
    return 1;
  }
  ah::Engine eng(0);
  std::string e;
  if (!eng.BuildHostOnly(ah::ep::RegionModel(c->model, *r), e)) {
    CopyOut("HIP EP: " + e, err, errlen);
    return 1;
  }
  CopyOut(eng.Describe(), buf, len);
  return 0;
}

int ah_ep_compile_region(const ah_ep_capability* c, int region, int device, ah_engine** out, char* err, int errlen) {
  const auto* r = EpRegion(c, region);
  if (!r || !out) {
    CopyOut("HIP EP: no such region", err, errlen);
    return 1;
  }
  if (!ah_ep_device_usable(device)) {
    CopyOut("HIP EP: device context is not initialized (device " + std::to_string(device) + ")", err, errlen);
    return 1;
  }
  auto h = std::make_unique<ah_engine>();
  h->eng = std::make_unique<ah::Engine>(device);
  std::string e;
  if (!h->eng->Build(ah::ep::RegionModel(c->model, *r), e)) {
    CopyOut("HIP EP: " + e, err, errlen);
    return 1;
  }
  *out = h.release();
  return 0;
}

void ah_ep_capability_destroy(ah_ep_capability* c) { delete c; }

// ---------------------------------------------------------------------------
// Host helpers
// ---------------------------------------------------------------------------
void ah_float_to_half_rne(const float* in, uint16_t* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = ah::FloatToHalfRNE(in[i]);
}

void ah_float_to_half_ftz(const float* in, uint16_t* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = ah::FloatToHalfFTZ(in[i]);
}

void ah_half_to_float(const uint16_t* in, float* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = ah::HalfToFloat(in[i]);
}

const char* ah_version(void) { return "arthip_b200 0.1.0 (sm_100a)"; }

}  // extern "C"
