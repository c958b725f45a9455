// The VapourSynth filter's loading path and frame IO (see vs_loader.h).
#include "vs_loader.h"

#include <cstring>
#include <unordered_map>
#include <vector>

#include "fp16_host.h"

namespace ah {
namespace vs {

namespace {

onnx::Node CastNode(const std::string& in, const std::string& out, const std::string& name, int to) {
  onnx::Node n;
  n.op_type = "Cast";
  n.name = name;
  n.inputs = {in};
  n.outputs = {out};
  onnx::Attribute a;
  a.name = "to";
  a.type = onnx::kAttrInt;
  a.i = to;
  a.has_i = true;
  n.attrs.push_back(a);
  return n;
}

// fp32 -> fp16 bits for one initializer, in place (raw_data, or float_data -> int32_data
// holding the halves, as the ONNX spec stores fp16 in int32_data).
void ConvertTensor(onnx::Tensor* t) {
  if (t->data_type != onnx::kFloat) return;
  t->data_type = onnx::kFloat16;
  if (!t->float_data.empty()) {
    t->int32_data.resize(t->float_data.size());
    for (size_t i = 0; i < t->float_data.size(); ++i) t->int32_data[i] = FloatToHalfFTZ(t->float_data[i]);
    t->float_data.clear();
  }
  if (t->has_raw) {
    const size_t n = t->raw_data.size() / sizeof(float);
    std::string out(n * sizeof(uint16_t), '\0');
    for (size_t i = 0; i < n; ++i) {
      float f;
      std::memcpy(&f, t->raw_data.data() + i * sizeof(float), sizeof(float));
      const uint16_t h = FloatToHalfFTZ(f);
      std::memcpy(&out[i * sizeof(uint16_t)], &h, sizeof(uint16_t));
    }
    t->raw_data.swap(out);
  }
}

}  // namespace

void ConvertFloatToFloat16(onnx::Model* m, const Fp16Options& opt, std::string* note) {
  onnx::Graph& g = m->graph;
  std::unordered_set<std::string> io_casts;       // names of the inserted boundary Casts
  std::unordered_set<std::string> io_keep_fp32;   // graph IO that keeps its fp32 type
  std::unordered_set<std::string> fp16_values;    // values known to be fp16 after conversion

  if (opt.cast_input) {
    int k = 0;
    std::vector<onnx::Node> front;
    for (const auto& in : g.inputs) {
      if (in.elem_type != onnx::kFloat) continue;
      const std::string cast = "graph_input_cast_" + std::to_string(k++);
      for (auto& n : g.nodes)
        for (auto& v : n.inputs)
          if (v == in.name) v = cast;
      front.push_back(CastNode(in.name, cast, cast, onnx::kFloat16));
      io_casts.insert(cast);
      io_keep_fp32.insert(in.name);
      fp16_values.insert(cast);
    }
    g.nodes.insert(g.nodes.begin(), front.begin(), front.end());
  }
  if (opt.cast_output) {
    int k = 0;
    for (const auto& out : g.outputs) {
      if (out.elem_type != onnx::kFloat) continue;
      const std::string cast = "graph_output_cast_" + std::to_string(k++);
      for (auto& n : g.nodes)
        for (auto& v : n.outputs)
          if (v == out.name) v = cast;
      g.nodes.push_back(CastNode(cast, out.name, cast, onnx::kFloat));
      io_casts.insert(cast);
      io_keep_fp32.insert(out.name);
      fp16_values.insert(cast);
    }
  }

  // Which nodes read each fp32 initializer: blocked (kept fp32) or converted.
  struct Use {
    bool fp32 = false, fp16 = false;
  };
  std::unordered_map<std::string, Use> fp32_inits;
  for (const auto& t : g.initializers)
    if (t.data_type == onnx::kFloat) fp32_inits[t.name];
  std::vector<size_t> blocked;
  for (size_t ni = 0; ni < g.nodes.size(); ++ni) {
    onnx::Node& n = g.nodes[ni];
    if (io_casts.count(n.name)) continue;
    const bool is_blocked = opt.op_block_list.count(n.op_type) != 0;
    for (const auto& v : n.inputs) {
      auto it = fp32_inits.find(v);
      if (it != fp32_inits.end()) (is_blocked ? it->second.fp32 : it->second.fp16) = true;
    }
    if (is_blocked) {
      blocked.push_back(ni);
    } else if (n.op_type == "Cast") {
      for (auto& a : n.attrs)
        if (a.name == "to" && a.i == onnx::kFloat) {
          a.i = onnx::kFloat16;
          break;
        }
    }
  }
  for (auto* list : {&g.inputs, &g.outputs})
    for (auto& v : *list)
      if (v.elem_type == onnx::kFloat && !io_keep_fp32.count(v.name)) {
        v.elem_type = onnx::kFloat16;
        fp16_values.insert(v.name);
      }
  for (auto& t : g.initializers) {
    auto it = fp32_inits.find(t.name);
    if (it == fp32_inits.end()) continue;
    // An initializer only blocked nodes read stays fp32 (unless forced), to keep its precision.
    if (opt.force_fp16_initializers || it->second.fp16) {
      ConvertTensor(&t);
      fp16_values.insert(t.name);
      if (it->second.fp32 && !opt.force_fp16_initializers && note)
        *note += "initializer '" + t.name + "' is used by both fp32 and fp16 nodes; ";
    }
  }
  // Blocked nodes run in fp32: Casts around their known-fp16 inputs and outputs.
  std::vector<onnx::Node> added;
  for (size_t ni : blocked) {
    onnx::Node& n = g.nodes[ni];
    for (size_t i = 0; i < n.inputs.size(); ++i) {
      if (!fp16_values.count(n.inputs[i])) continue;
      const std::string renamed = n.name + "_input_cast_" + std::to_string(i);
      added.push_back(CastNode(n.inputs[i], renamed, n.name + "_input_cast" + std::to_string(i), onnx::kFloat));
      n.inputs[i] = renamed;
    }
    for (size_t i = 0; i < n.outputs.size(); ++i) {
      if (!fp16_values.count(n.outputs[i])) continue;
      const std::string renamed = n.name + "_output_cast_" + std::to_string(i);
      added.push_back(
          CastNode(renamed, n.outputs[i], n.name + "_output_cast" + std::to_string(i), onnx::kFloat16));
      n.outputs[i] = renamed;
    }
  }
  // Appended after the graph's nodes, as the reference does; the engine's parse and the
  // partitioner resolve values by name.
  g.nodes.insert(g.nodes.end(), added.begin(), added.end());
}

bool SpecifyShape(onnx::Model* m, int64_t tile_w, int64_t tile_h, int64_t batch, std::string* err) {
  onnx::Graph& g = m->graph;
  if (g.inputs.size() != 1) {
    *err = "graph must have a single input";
    return false;
  }
  if (g.outputs.size() != 1) {
    *err = "graph must have a single output";
    return false;
  }
  auto& in = g.inputs[0].dims;
  if (in.size() != 4) {
    *err = "input dimension must be 4";
    return false;
  }
  in[0] = batch;
  in[2] = tile_h;
  in[3] = tile_w;
  auto& out = g.outputs[0].dims;
  if (out.size() != 4) {
    *err = "output dimension must be 4";
    return false;
  }
  out[0] = batch;
  out[2] = -1;
  out[3] = -1;
  return true;
}

std::string ValidateClipFormat(const ClipFormat& f) {
  if (f.color_family != kCfGray && f.color_family != kCfYUV && f.color_family != kCfRGB)
    return "expects a gray, YUV or RGB clip";
  const bool ok = (f.sample_type == kStInteger && (f.bits_per_sample == 8 || f.bits_per_sample == 16)) ||
                  (f.sample_type == kStFloat && (f.bits_per_sample == 16 || f.bits_per_sample == 32));
  if (!ok) return "expects 8/16-bit int or fp16/fp32 float input";
  if (f.subsampling_w != 0 || f.subsampling_h != 0)
    return "subsampled input (YUV420/YUV422) is not supported; convert to 4:4:4 first";
  return "";
}

std::string ValidateTiling(const ModelArgs& a, const ClipFormat& clip) {
  const int64_t ow = a.overlap_n >= 1 ? a.overlap[0] : 0;
  const int64_t oh = a.overlap_n >= 2 ? a.overlap[1] : ow;
  if (ow < 0 || oh < 0) return "\"overlap\" must be non-negative";
  if (ow != 0 || oh != 0)
    return "\"overlap\" is not supported: this filter always processes the whole frame in one tile";
  if (a.tilesize_n >= 1) {
    const int64_t tw = a.tilesize[0];
    const int64_t th = a.tilesize_n >= 2 ? a.tilesize[1] : tw;
    if (tw != clip.width || th != clip.height)
      return "\"tilesize\" is not supported: this filter always processes the whole frame in one tile";
  }
  return "";
}

std::string ValidateChannels(const ClipFormat& f, int model_in_channels) {
  if (model_in_channels > 3)
    return "model requires " + std::to_string(model_in_channels) +
           " input channels, but a clip provides at most 3 full-resolution planes";
  if (f.num_planes != model_in_channels)
    return "clip has " + std::to_string(f.num_planes) + " plane(s) but the model expects " +
           std::to_string(model_in_channels) + " input channel(s)";
  return "";
}

void PackPlanes(const ClipFormat& f, const void* const* planes, const ptrdiff_t* strides, bool to_fp32,
                void* dst) {
  const size_t plane = static_cast<size_t>(f.width) * f.height;
  float* d32 = to_fp32 ? static_cast<float*>(dst) : nullptr;
  uint16_t* d16 = to_fp32 ? nullptr : static_cast<uint16_t*>(dst);
  for (int c = 0; c < f.num_planes; ++c) {
    const uint8_t* base = static_cast<const uint8_t*>(planes[c]);
    for (int y = 0; y < f.height; ++y) {
      const uint8_t* row = base + static_cast<ptrdiff_t>(y) * strides[c];
      const size_t o = c * plane + static_cast<size_t>(y) * f.width;
      if (f.sample_type == kStFloat && f.bits_per_sample == 16 && !to_fp32) {
        std::memcpy(d16 + o, row, static_cast<size_t>(f.width) * 2);  // same type and layout
        continue;
      }
      if (f.sample_type == kStFloat && f.bits_per_sample == 32 && to_fp32) {
        std::memcpy(d32 + o, row, static_cast<size_t>(f.width) * 4);
        continue;
      }
      for (int x = 0; x < f.width; ++x) {
        float v;
        if (f.sample_type == kStInteger) {
          v = f.bits_per_sample == 8 ? row[x] * (1.0f / 255.0f)
                                     : reinterpret_cast<const uint16_t*>(row)[x] * (1.0f / 65535.0f);
        } else if (f.bits_per_sample == 16) {
          v = HalfToFloat(reinterpret_cast<const uint16_t*>(row)[x]);
        } else {
          v = reinterpret_cast<const float*>(row)[x];
        }
        if (to_fp32) d32[o + x] = v;
        else d16[o + x] = FloatToHalfRNE(v);
      }
    }
  }
}

void UnpackPlanes(const void* src, bool src_fp32, int out_w, int out_h, void* const* dst_planes,
                  const ptrdiff_t* dst_strides, int n_planes, bool as_int16) {
  const size_t plane = static_cast<size_t>(out_w) * out_h;
  for (int c = 0; c < n_planes; ++c) {
    uint8_t* base = static_cast<uint8_t*>(dst_planes[c]);
    for (int y = 0; y < out_h; ++y) {
      uint8_t* row = base + static_cast<ptrdiff_t>(y) * dst_strides[c];
      const size_t o = c * plane + static_cast<size_t>(y) * out_w;
      if (src_fp32) {
        std::memcpy(row, static_cast<const float*>(src) + o, static_cast<size_t>(out_w) * 4);
      } else if (!as_int16) {
        std::memcpy(row, static_cast<const uint16_t*>(src) + o, static_cast<size_t>(out_w) * 2);
      } else {
        const uint16_t* s = static_cast<const uint16_t*>(src) + o;
        uint16_t* r = reinterpret_cast<uint16_t*>(row);
        for (int x = 0; x < out_w; ++x) {
          // Clamped first: a float outside [0, 65535] has no defined uint16 conversion.
          const float v = HalfToFloat(s[x]) * 65535.0f + 0.5f;
          r[x] = static_cast<uint16_t>(v > 0.f ? (v < 65535.f ? v : 65535.f) : 0.f);
        }
      }
    }
  }
}

}  // namespace vs
}  // namespace ah
