// The VapourSynth filter hip.Model as plain C (no VapourSynth headers): creation-time
// validation, model loading and fp16 conversion, the engine pool, and frame processing on
// plane pointers. A plugin shim registers the function with VapourSynth and maps its frames
// and maps onto these calls (ah_vs_* in include/arthip_b200.h). Follows hipCreate /
// hipGetFrame (src/vapoursynth/vs_hip.cpp:77-591); every error is prefixed "hip.Model: ".
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "../../include/arthip_b200.h"
#include "engine.h"
#include "vs_loader.h"

struct ah_vs_model {
  std::vector<std::unique_ptr<ah::Engine>> engines;
  std::atomic<unsigned> next{0};
  bool output_fp16 = true;
  bool output_fp32 = false;
  int input_channels = 1;
  int output_channels = 1;
  bool flexible = false;
  ah_vs_format out_format{};
};

namespace {

void CopyPlain(const std::string& s, char* dst, int len) {
  if (!dst || len <= 0) return;
  size_t n = s.size();
  if (n > static_cast<size_t>(len) - 1) n = static_cast<size_t>(len) - 1;
  std::memcpy(dst, s.data(), n);
  dst[n] = '\0';
}

void CopyErr(const std::string& s, char* dst, int len) { CopyPlain("hip.Model: " + s, dst, len); }

ah::vs::ClipFormat ToClip(const ah_vs_format& f) {
  ah::vs::ClipFormat c;
  c.color_family = f.color_family;
  c.sample_type = f.sample_type;
  c.bits_per_sample = f.bits_per_sample;
  c.subsampling_w = f.subsampling_w;
  c.subsampling_h = f.subsampling_h;
  c.num_planes = f.num_planes;
  c.width = f.width;
  c.height = f.height;
  return c;
}

bool LoadModel(const void* bytes, size_t size, const char* path, ah::onnx::Model* m, std::string* err) {
  if (bytes) {
    if (!ah::onnx::ParseModel(static_cast<const uint8_t*>(bytes), size, m, err)) {
      *err = "parse onnx serialization failed";
      return false;
    }
    return true;
  }
  if (!path) {
    *err = "no network_path given";
    return false;
  }
  if (!ah::onnx::LoadModelFile(path, m, err)) {
    *err = std::string("parse ") + path + " failed";
    return false;
  }
  return true;
}

// Copy-out convention of the byte-returning calls: out == NULL asks for the size only; a
// buffer smaller than the result is an error (return 1, nothing written).
int PutBytes(const std::string& s, void* out, size_t cap, size_t* out_bytes, char* err, int errlen) {
  if (out_bytes) *out_bytes = s.size();
  if (!out) return 0;
  if (cap < s.size()) {
    CopyPlain("output buffer too small (" + std::to_string(s.size()) + " bytes needed)", err, errlen);
    return 1;
  }
  std::memcpy(out, s.data(), s.size());
  return 0;
}

}  // namespace

extern "C" {

int ah_convert_float_to_float16(const void* model, size_t model_bytes, int force_fp16_initializers,
                                const char* op_block_list, int cast_input, int cast_output, void* out, size_t cap,
                                size_t* out_bytes, char* err, int errlen) {
  ah::onnx::Model m;
  std::string e;
  if (!model || !ah::onnx::ParseModel(static_cast<const uint8_t*>(model), model_bytes, &m, &e)) {
    CopyPlain("parse onnx serialization failed", err, errlen);
    return 1;
  }
  ah::vs::Fp16Options o;
  o.force_fp16_initializers = force_fp16_initializers != 0;
  o.cast_input = cast_input != 0;
  o.cast_output = cast_output != 0;
  if (op_block_list) {
    std::string cur;
    for (const char* p = op_block_list;; ++p) {
      if (*p == ',' || *p == '\0') {
        if (!cur.empty()) o.op_block_list.insert(cur);
        cur.clear();
        if (*p == '\0') break;
      } else {
        cur.push_back(*p);
      }
    }
  }
  std::string note;
  ah::vs::ConvertFloatToFloat16(&m, o, &note);
  return PutBytes(ah::onnx::EncodeModel(m), out, cap, out_bytes, err, errlen);
}

int ah_load_onnx(const void* model, size_t model_bytes, const char* path, int64_t tile_w, int64_t tile_h, void* out,
                 size_t cap, size_t* out_bytes, char* err, int errlen) {
  ah::onnx::Model m;
  std::string e;
  if (!LoadModel(model, model_bytes, path, &m, &e) || !ah::vs::SpecifyShape(&m, tile_w, tile_h, 1, &e)) {
    CopyPlain(e, err, errlen);
    return 1;
  }
  return PutBytes(ah::onnx::EncodeModel(m), out, cap, out_bytes, err, errlen);
}

int ah_vs_model_create(const ah_vs_format* clip, const void* model, size_t model_bytes, const char* network_path,
                       const ah_vs_args* args, ah_vs_model** out, char* err, int errlen) {
  if (!clip || !args || !out) {
    CopyErr("invalid arguments", err, errlen);
    return 1;
  }
  const ah::vs::ClipFormat cf = ToClip(*clip);
  std::string e = ah::vs::ValidateClipFormat(cf);
  if (!e.empty()) {
    CopyErr(e, err, errlen);
    return 1;
  }
  ah::vs::ModelArgs a;
  a.device_id = args->device_id;
  a.num_streams = args->num_streams < 1 ? 1 : args->num_streams;
  a.overlap_n = args->overlap_n;
  a.overlap[0] = args->overlap[0];
  a.overlap[1] = args->overlap[1];
  a.tilesize_n = args->tilesize_n;
  a.tilesize[0] = args->tilesize[0];
  a.tilesize[1] = args->tilesize[1];
  e = ah::vs::ValidateTiling(a, cf);
  if (!e.empty()) {
    CopyErr(e, err, errlen);
    return 1;
  }
  auto d = std::make_unique<ah_vs_model>();
  d->output_fp16 = args->fp16_set ? args->fp16 != 0 : true;  // fp16 defaults to true
  d->flexible = args->flexible_output_prop && args->flexible_output_prop[0] != '\0';

  ah::onnx::Model m;
  if (!LoadModel(model, model_bytes, network_path, &m, &e) || !ah::vs::SpecifyShape(&m, 0, 0, 1, &e)) {
    CopyErr(e, err, errlen);
    return 1;
  }
  // fp16 = true converts an fp32 model at load time. An fp32 clip keeps fp32 IO on both
  // ends: the inserted boundary Casts fold into the engine's device-side IO conversions.
  if (d->output_fp16) {
    const bool clip_fp32 = cf.sample_type == ah::vs::kStFloat && cf.bits_per_sample == 32;
    ah::vs::Fp16Options o;
    o.force_fp16_initializers = true;
    o.cast_input = clip_fp32;
    o.cast_output = clip_fp32;
    std::string note;
    ah::vs::ConvertFloatToFloat16(&m, o, &note);
  }
  for (int i = 0; i < a.num_streams; ++i) {
    auto eng = std::make_unique<ah::Engine>(a.device_id);
    if (!eng->Build(m, e)) {
      CopyErr(e, err, errlen);
      return 1;
    }
    d->engines.push_back(std::move(eng));
  }
  ah::Engine& e0 = *d->engines[0];
  d->output_fp32 = e0.OutputIsFp32();
  d->input_channels = std::max(1, e0.InputChannels());
  e = ah::vs::ValidateChannels(cf, d->input_channels);
  if (!e.empty()) {
    CopyErr(e, err, errlen);
    return 1;
  }
  std::vector<int64_t> probe_in{1, d->input_channels, 64, 64}, probe_out;
  if (!e0.GetOutputShape(probe_in, probe_out) || probe_out.size() != 4) {
    CopyErr("model shape probe failed", err, errlen);
    return 1;
  }
  // The published plane count is the graph's final output channels (after a trailing
  // DepthToSpace), not the tail conv's.
  d->output_channels = std::max<int>(1, static_cast<int>(probe_out[1]));
  const int scale_w = static_cast<int>(probe_out[3] / probe_in[3]);
  const int scale_h = static_cast<int>(probe_out[2] / probe_in[2]);
  ah_vs_format& o = d->out_format;
  o = *clip;
  o.width = clip->width * scale_w;
  o.height = clip->height * scale_h;
  // A 3-channel output without the flexible protocol is an RGB frame; otherwise gray.
  o.color_family = (d->output_channels == 3 && !d->flexible) ? ah::vs::kCfRGB : ah::vs::kCfGray;
  o.sample_type = (d->output_fp32 || d->output_fp16) ? ah::vs::kStFloat : ah::vs::kStInteger;
  o.bits_per_sample = d->output_fp32 ? 32 : 16;
  o.subsampling_w = o.subsampling_h = 0;
  o.num_planes = o.color_family == ah::vs::kCfRGB ? 3 : 1;
  *out = d.release();
  return 0;
}

int ah_vs_model_output(const ah_vs_model* m, ah_vs_format* out_format, int* num_output_channels) {
  if (!m) return 1;
  if (out_format) *out_format = m->out_format;
  if (num_output_channels) *num_output_channels = m->output_channels;
  return 0;
}

int ah_vs_model_get_frame(ah_vs_model* m, const ah_vs_format* f, const void* const* src_planes,
                          const ptrdiff_t* src_strides, void* const* dst_planes, const ptrdiff_t* dst_strides,
                          int n_dst_planes, char* err, int errlen) {
  if (!m || !f || !src_planes || !src_strides || (n_dst_planes > 0 && (!dst_planes || !dst_strides))) {
    CopyErr("invalid frame arguments", err, errlen);
    return 1;
  }
  // Per frame (variable-format clips): every plane full size, plane count = model channels.
  if (f->subsampling_w != 0 || f->subsampling_h != 0) {
    CopyErr("subsampled input frame: every plane must have the luma plane's dimensions", err, errlen);
    return 1;
  }
  const int in_c = f->num_planes;
  if (in_c != m->input_channels || in_c > 3) {
    CopyErr("input clip plane count does not match the model's input channels", err, errlen);
    return 1;
  }
  // Round-robin over the engine pool; each engine serialises its own calls.
  ah::Engine& eng = *m->engines[m->next.fetch_add(1) % m->engines.size()];
  std::vector<int64_t> in_shape{1, in_c, f->height, f->width}, out_shape;
  if (!eng.GetOutputShape(in_shape, out_shape) || out_shape.size() != 4) {
    CopyErr("shape propagation failed", err, errlen);
    return 1;
  }
  const int out_c = static_cast<int>(out_shape[1]);
  const int out_h = static_cast<int>(out_shape[2]);
  const int out_w = static_cast<int>(out_shape[3]);
  const bool host_fp32 = eng.InputIsFp32();
  const size_t in_elems = static_cast<size_t>(f->width) * f->height * in_c;
  std::vector<uint8_t> in_pack(in_elems * (host_fp32 ? 4 : 2));
  ah::vs::PackPlanes(ToClip(*f), src_planes, src_strides, host_fp32, in_pack.data());
  const size_t out_elems = static_cast<size_t>(out_w) * out_h * out_c;
  std::vector<uint8_t> out_pack(out_elems * (m->output_fp32 ? 4 : 2));
  std::string e;
  if (!eng.Run(in_pack.data(), in_shape, out_pack.data(), e)) {
    CopyErr(e, err, errlen);
    return 2;
  }
  ah::vs::UnpackPlanes(out_pack.data(), m->output_fp32, out_w, out_h, dst_planes, dst_strides,
                       std::min(n_dst_planes, out_c), !m->output_fp32 && !m->output_fp16);
  return 0;
}

void ah_vs_model_destroy(ah_vs_model* m) { delete m; }

int ah_device_properties(int device, char* name, int namelen, int64_t* pci_device_id, int64_t* clock_rate_khz,
                         int64_t* global_memory) {
  cudaDeviceProp p;
  if (cudaGetDeviceProperties(&p, device) != cudaSuccess) {
    (void)cudaGetLastError();
    return 1;
  }
  CopyPlain(p.name, name, namelen);
  if (pci_device_id) *pci_device_id = p.pciDeviceID;
  if (clock_rate_khz) {
    int khz = 0;
    cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, device);
    *clock_rate_khz = khz;
  }
  if (global_memory) *global_memory = static_cast<int64_t>(p.totalGlobalMem);
  return 0;
}

}  // extern "C"
