// Engine core: ONNX parse and fusion, shape propagation, per-resolution device plan,
// frame execution. See engine.h for the contract.
#include "engine.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <numeric>
#include <sstream>
#include <unordered_set>

#include "fp16_host.h"

namespace ah {

namespace {

bool EnvOn(const char* name) {
  const char* e = std::getenv(name);
  return e && *e == '1';
}

int64_t Numel(const std::vector<int64_t>& s) {
  return std::accumulate(s.begin(), s.end(), int64_t{1}, std::multiplies<int64_t>());
}

size_t DtypeSize(int dt) {
  switch (dt) {
    case onnx::kFloat: return 4;
    case onnx::kFloat16: return 2;
    case onnx::kDouble: return 8;
    case onnx::kInt64: return 8;
    case onnx::kInt32:
    case onnx::kUint32: return 4;
    case onnx::kInt16:
    case onnx::kUint16:
    case onnx::kBfloat16: return 2;
    case onnx::kInt8:
    case onnx::kUint8:
    case onnx::kBool: return 1;
    default: return 0;
  }
}

// Initializer bytes with the declared dtype preserved. FLOAT16 values stored in
// int32_data are 16-bit bit patterns, one slot per element (the ONNX schema; the
// reference reads them the same way, hip_engine.cc:88-103).
bool Materialize(const onnx::Tensor& t, WeightSpec* w, std::string& err) {
  w->dtype = t.data_type;
  w->shape = t.dims;
  w->data.clear();
  if (t.external) {
    err = "initializer '" + t.name + "' uses external data, which is not supported";
    return false;
  }
  const size_t es = DtypeSize(t.data_type);
  if (t.has_raw && !t.raw_data.empty()) {
    if (es == 0) {
      err = "initializer '" + t.name + "' has an unsupported dtype";
      return false;
    }
    w->data.assign(t.raw_data.begin(), t.raw_data.end());
    return true;
  }
  if (!t.float_data.empty()) {
    if (t.data_type != onnx::kFloat) {
      err = "initializer '" + t.name + "' has float_data with a non-FLOAT dtype";
      return false;
    }
    w->data.resize(t.float_data.size() * 4);
    std::memcpy(w->data.data(), t.float_data.data(), w->data.size());
  } else if (!t.double_data.empty()) {
    if (t.data_type != onnx::kDouble) {
      err = "initializer '" + t.name + "' has double_data with a non-DOUBLE dtype";
      return false;
    }
    w->data.resize(t.double_data.size() * 8);
    std::memcpy(w->data.data(), t.double_data.data(), w->data.size());
  } else if (!t.int32_data.empty()) {
    if (es == 0) {
      err = "initializer '" + t.name + "' has an unsupported dtype";
      return false;
    }
    w->data.resize(t.int32_data.size() * es);
    for (size_t k = 0; k < t.int32_data.size(); ++k) {
      const uint32_t v = static_cast<uint32_t>(t.int32_data[k]);
      std::memcpy(w->data.data() + k * es, &v, es);  // little-endian low bytes
    }
  } else if (!t.int64_data.empty()) {
    w->data.resize(t.int64_data.size() * 8);
    std::memcpy(w->data.data(), t.int64_data.data(), w->data.size());
  }
  return true;
}

float WeightAt(const WeightSpec& w, size_t i) {
  if (w.dtype == onnx::kFloat) {
    if ((i + 1) * 4 > w.data.size()) return 0.f;
    float v;
    std::memcpy(&v, w.data.data() + i * 4, 4);
    return v;
  }
  if (w.dtype == onnx::kFloat16) {
    if ((i + 1) * 2 > w.data.size()) return 0.f;
    uint16_t b;
    std::memcpy(&b, w.data.data() + i * 2, 2);
    return HalfToFloat(b);
  }
  if (w.dtype == onnx::kDouble) {
    if ((i + 1) * 8 > w.data.size()) return 0.f;
    double v;
    std::memcpy(&v, w.data.data() + i * 8, 8);
    return static_cast<float>(v);
  }
  return 0.f;
}

// Weight element as fp16 bits: fp16 storage is used verbatim, fp32 is rounded RNE.
uint16_t WeightHalf(const WeightSpec& w, size_t i) {
  if (w.dtype == onnx::kFloat16) {
    uint16_t b = 0;
    if ((i + 1) * 2 <= w.data.size()) std::memcpy(&b, w.data.data() + i * 2, 2);
    return b;
  }
  return FloatToHalfRNE(WeightAt(w, i));
}

}  // namespace

const char* OpTypeName(OpType t) {
  switch (t) {
    case OpType::Conv: return "Conv";
    case OpType::Sigmoid: return "Sigmoid";
    case OpType::Mul: return "Mul";
    case OpType::Add: return "Add";
    case OpType::Clip: return "Clip";
    case OpType::Relu: return "Relu";
    case OpType::DepthToSpace: return "DepthToSpace";
  }
  return "?";
}

Engine::Engine(int device_id) : device_id_(device_id) {
  prof_ = EnvOn("VSHIP_PROFILE");
  trace_ = EnvOn("VSHIP_TRACE");
  poison_ = EnvOn("VSHIP_POISON");
  sync_each_ = EnvOn("VSHIP_SYNC_EACH");
  no_graph_ = EnvOn("ARTHIP_NO_GRAPH") || prof_ || poison_ || sync_each_;
  // Conv algorithm for 64 -> 64 layers: "winograd" opts into the Winograd kernel (the
  // reference's numerics); anything else keeps the direct implicit GEMM. Read once here.
  if (const char* a = std::getenv("ARTHIP_CONV_ALGO")) conv_algo_ = std::string(a) == "winograd" ? 1 : 0;
}

Engine::~Engine() { DestroyAll(); }

bool Engine::SetDevice(std::string& error) const {
  cudaError_t e = cudaSetDevice(device_id_);
  if (e != cudaSuccess) {
    error = "cudaSetDevice(" + std::to_string(device_id_) + ") failed: " + cudaGetErrorString(e);
    (void)cudaGetLastError();
    return false;
  }
  return true;
}

// ---------------------------------------------------------------------------
// Parse + fuse
// ---------------------------------------------------------------------------
bool Engine::BuildHostOnly(const onnx::Model& model, std::string& error) { return Parse(model, error); }

bool Engine::Build(const onnx::Model& model, std::string& error) {
  if (!Parse(model, error)) return false;
  if (!SetDevice(error)) return false;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device_id_) == cudaSuccess && sms > 0)
    num_sms_ = sms;
  if (!stream_) {
    cudaError_t e = cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
      error = std::string("cudaStreamCreate failed: ") + cudaGetErrorString(e);
      return false;
    }
  }
  if (!status_) {
    cudaError_t e = cudaMalloc(&status_, sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMemset(status_, 0, sizeof(uint32_t));
    if (e != cudaSuccess) {
      error = std::string("cudaMalloc of the status word failed: ") + cudaGetErrorString(e);
      return false;
    }
  }
  device_ready_ = true;
  return true;
}

bool Engine::Parse(const onnx::Model& model, std::string& error) {
  const onnx::Graph& g = model.graph;
  ops_.clear();
  weights_.clear();
  input_is_fp32_ = output_is_fp32_ = false;
  if (g.inputs.empty() || g.outputs.empty()) {
    error = "model must have at least one input and output";
    return false;
  }
  input_name_ = g.inputs[0].name;
  output_name_ = g.outputs[0].name;
  for (size_t i = 0; i < g.initializers.size(); ++i) {
    const onnx::Tensor& t = g.initializers[i];
    if (t.name.empty()) {
      error = "initializer #" + std::to_string(i) + " has no name";
      return false;
    }
    if (!Materialize(t, &weights_[t.name], error)) return false;
  }

  std::unordered_map<std::string, std::vector<int>> consumers;
  for (int ni = 0; ni < static_cast<int>(g.nodes.size()); ++ni)
    for (const auto& in : g.nodes[ni].inputs)
      if (!in.empty()) consumers[in].push_back(ni);
  auto users = [&](const std::string& t) -> const std::vector<int>& {
    static const std::vector<int> none;
    auto it = consumers.find(t);
    return it == consumers.end() ? none : it->second;
  };
  std::unordered_set<std::string> protected_out;
  for (const auto& o : g.outputs) protected_out.insert(o.name);
  // `t` can be renamed away by a fusion only when every consumer is in `allowed` and it
  // is not a value the graph must still produce.
  auto only_used_by = [&](const std::string& t, std::initializer_list<int> allowed) {
    if (t == output_name_ || protected_out.count(t)) return false;
    for (int c : users(t)) {
      bool ok = false;
      for (int a : allowed) ok = ok || (a == c);
      if (!ok) return false;
    }
    return true;
  };
  auto scalar_bound = [&](const std::string& name, float& dst) -> bool {
    if (name.empty()) return true;
    auto it = weights_.find(name);
    if (it == weights_.end()) {
      error = "Clip bound '" + name + "' is not an initializer; dynamic Clip bounds are not supported";
      return false;
    }
    const WeightSpec& w = it->second;
    if (w.data.empty()) return true;
    if ((w.dtype == onnx::kFloat && w.data.size() >= 4) || (w.dtype == onnx::kFloat16 && w.data.size() >= 2) ||
        (w.dtype == onnx::kDouble && w.data.size() >= 8)) {
      dst = WeightAt(w, 0);
      return true;
    }
    error = "Clip bound initializer '" + name + "' has an unsupported dtype or truncated storage";
    return false;
  };

  // Boundary Cast folding: fp32 graph IO around an fp16 body.
  std::vector<bool> consumed(g.nodes.size(), false);
  if (g.inputs[0].elem_type == onnx::kFloat) {
    input_is_fp32_ = true;
    for (size_t ni = 0; ni < g.nodes.size(); ++ni) {
      const auto& n = g.nodes[ni];
      if (n.op_type == "Cast" && !n.inputs.empty() && n.inputs[0] == input_name_ && !n.outputs.empty()) {
        input_name_ = n.outputs[0];
        consumed[ni] = true;
        break;
      }
    }
  }
  if (g.outputs[0].elem_type == onnx::kFloat) {
    output_is_fp32_ = true;
    for (size_t ni = 0; ni < g.nodes.size(); ++ni) {
      const auto& n = g.nodes[ni];
      if (n.op_type == "Cast" && !n.outputs.empty() && n.outputs[0] == output_name_ && !n.inputs.empty()) {
        output_name_ = n.inputs[0];
        consumed[ni] = true;
        break;
      }
    }
  }

  for (size_t ni = 0; ni < g.nodes.size(); ++ni) {
    if (consumed[ni]) continue;
    const onnx::Node& n = g.nodes[ni];
    if (n.outputs.empty() || n.outputs[0].empty()) continue;
    auto in = [&](size_t i) { return i < n.inputs.size() ? n.inputs[i] : std::string(); };
    OpSpec op;
    op.out = n.outputs[0];
    const std::string& t = n.op_type;
    if (t == "Conv") {
      op.type = OpType::Conv;
      op.in0 = in(0);
      op.in1 = in(1);
      op.bias = in(2);
      if (op.in0.empty() || op.in1.empty()) {
        error = "Conv missing inputs";
        return false;
      }
      int sh = 1, sw = 1, dh = 1, dw = 1, grp = 1;
      bool pad1 = false;
      if (auto a = n.attr("strides"); a && a->ints.size() >= 2) sh = a->ints[0], sw = a->ints[1];
      if (auto a = n.attr("dilations"); a && a->ints.size() >= 2) dh = a->ints[0], dw = a->ints[1];
      if (auto a = n.attr("group")) grp = static_cast<int>(a->i);
      if (auto a = n.attr("auto_pad")) {
        if (a->s == "SAME_UPPER" || a->s == "SAME_LOWER") pad1 = true;
        else if (a->s != "VALID" && a->s != "NOTSET") {
          error = "unsupported Conv auto_pad '" + a->s + "'";
          return false;
        }
      }
      if (auto a = n.attr("pads"); a && !a->ints.empty()) {
        // ONNX order [top, left, bottom, right]: only symmetric 1-padding is a 3x3 SAME conv.
        if (a->ints.size() != 4 || a->ints[0] != 1 || a->ints[1] != 1 || a->ints[2] != 1 || a->ints[3] != 1) {
          error = "unsupported Conv pads (only symmetric 1-padding on both axes is supported)";
          return false;
        }
        pad1 = true;
      }
      if (sh != 1 || sw != 1 || dh != 1 || dw != 1 || grp != 1 || !pad1) {
        error = "unsupported Conv configuration (only 3x3 stride 1, pad 1 supported)";
        return false;
      }
      auto wit = weights_.find(op.in1);
      if (wit == weights_.end()) {
        error = "expected initializer '" + op.in1 + "' was not found";
        return false;
      }
      const WeightSpec& ws = wit->second;
      if (ws.shape.size() != 4) {
        error = "Conv weight '" + op.in1 + "' must be a rank-4 tensor";
        return false;
      }
      if (ws.shape[2] != 3 || ws.shape[3] != 3) {
        error = "Conv weight '" + op.in1 + "' must be 3x3 (got " + std::to_string(ws.shape[2]) + "x" +
                std::to_string(ws.shape[3]) + ")";
        return false;
      }
      if (ws.shape[0] <= 0 || ws.shape[1] <= 0) {
        error = "Conv weight '" + op.in1 + "' has a non-positive channel count";
        return false;
      }
      if (ws.shape[0] > 256) {
        error = "conv supports at most 256 output channels (got " + std::to_string(ws.shape[0]) + ")";
        return false;
      }
      if (ws.shape[1] > 256) {
        error = "conv supports at most 256 input channels (got " + std::to_string(ws.shape[1]) + ")";
        return false;
      }
      if (ws.dtype != onnx::kFloat && ws.dtype != onnx::kFloat16) {
        error = "Conv weight '" + op.in1 + "' has unsupported dtype " + std::to_string(ws.dtype);
        return false;
      }
      const size_t need = static_cast<size_t>(Numel(ws.shape)) * DtypeSize(ws.dtype);
      if (ws.data.size() < need) {
        error = "Conv weight '" + op.in1 + "' storage is truncated (" + std::to_string(ws.data.size()) +
                " bytes, need " + std::to_string(need) + ")";
        return false;
      }
      if (!op.bias.empty()) {
        auto bit = weights_.find(op.bias);
        if (bit == weights_.end()) {
          error = "expected initializer '" + op.bias + "' was not found";
          return false;
        }
        const WeightSpec& bs = bit->second;
        if (bs.shape.size() != 1 || bs.shape[0] != ws.shape[0]) {
          error = "Conv bias '" + op.bias + "' must be a rank-1 tensor with the weight's channel count";
          return false;
        }
        if (bs.dtype != onnx::kFloat && bs.dtype != onnx::kFloat16) {
          error = "Conv bias '" + op.bias + "' has unsupported dtype " + std::to_string(bs.dtype);
          return false;
        }
        if (bs.data.size() < static_cast<size_t>(bs.shape[0]) * DtypeSize(bs.dtype)) {
          error = "Conv bias '" + op.bias + "' storage is truncated";
          return false;
        }
      }
      // Epilogue fusion. SiLU = Mul(x, Sigmoid(x)); the conv output is renamed to the
      // Mul's output, so it must have no other consumer and not be a graph output.
      const std::string conv_out = op.out;
      bool fused = false;
      for (int ci : users(conv_out)) {
        const onnx::Node& c = g.nodes[ci];
        if (consumed[ci]) continue;
        if (c.op_type == "Sigmoid" && !c.outputs.empty()) {
          const std::string& s_out = c.outputs[0];
          for (int ci2 : users(s_out)) {
            const onnx::Node& m = g.nodes[ci2];
            if (m.op_type != "Mul" || m.inputs.size() != 2 || m.outputs.empty()) continue;
            const bool pair = (m.inputs[0] == conv_out && m.inputs[1] == s_out) ||
                              (m.inputs[0] == s_out && m.inputs[1] == conv_out);
            if (!pair) continue;
            if (!only_used_by(conv_out, {ci, ci2}) || !only_used_by(s_out, {ci2})) continue;
            op.act = kActSilu;
            op.out = m.outputs[0];
            consumed[ci] = consumed[ci2] = true;
            fused = true;
            break;
          }
        } else if (c.op_type == "Relu" && !c.outputs.empty()) {
          if (!only_used_by(conv_out, {ci})) continue;
          op.act = kActRelu;
          op.out = c.outputs[0];
          consumed[ci] = true;
          fused = true;
        }
        if (fused) break;
      }
    } else if (t == "Sigmoid") {
      op.type = OpType::Sigmoid;
      op.in0 = in(0);
    } else if (t == "Relu") {
      op.type = OpType::Relu;
      op.in0 = in(0);
    } else if (t == "Mul") {
      op.type = OpType::Mul;
      op.in0 = in(0);
      op.in1 = in(1);
    } else if (t == "Add") {
      op.type = OpType::Add;
      op.in0 = in(0);
      op.in1 = in(1);
    } else if (t == "Clip") {
      op.type = OpType::Clip;
      op.in0 = in(0);
      // An omitted bound means the element type's extremum, never 0 or 1.
      if (auto a = n.attr("min")) op.clip_min = a->f;
      if (auto a = n.attr("max")) op.clip_max = a->f;
      if (!scalar_bound(in(1), op.clip_min)) return false;
      if (!scalar_bound(in(2), op.clip_max)) return false;
    } else if (t == "DepthToSpace") {
      op.type = OpType::DepthToSpace;
      op.in0 = in(0);
      if (auto a = n.attr("blocksize")) op.blocksize = static_cast<int>(a->i);
      if (op.blocksize < 1) {
        error = "DepthToSpace blocksize must be positive";
        return false;
      }
      if (auto a = n.attr("mode"); a && a->s != "DCR") {
        error = "only DepthToSpace mode DCR is supported";
        return false;
      }
      for (int ci : users(op.out)) {
        const onnx::Node& c = g.nodes[ci];
        if (c.op_type != "Clip" || consumed[ci] || c.outputs.empty()) continue;
        if (!only_used_by(op.out, {ci})) continue;
        if (auto a = c.attr("min")) op.clip_min = a->f;
        if (auto a = c.attr("max")) op.clip_max = a->f;
        if (!scalar_bound(c.inputs.size() > 1 ? c.inputs[1] : std::string(), op.clip_min)) return false;
        if (!scalar_bound(c.inputs.size() > 2 ? c.inputs[2] : std::string(), op.clip_max)) return false;
        op.fuse_clip = true;
        consumed[ci] = true;
        op.out = c.outputs[0];
        break;
      }
    } else {
      error = "unsupported op '" + t + "' in fused graph";
      return false;
    }
    ops_.push_back(std::move(op));
  }

  // Residual Add fusion: an Add whose later-produced operand is a Conv output with no
  // other reader becomes that conv's epilogue add (up to two per conv: the block
  // residual and the global skip). Repeat until nothing changes, since a fused conv's
  // renamed output can feed the next Add.
  for (bool changed = true; changed;) {
    changed = false;
    std::unordered_map<std::string, size_t> producer;
    for (size_t i = 0; i < ops_.size(); ++i) producer[ops_[i].out] = i;
    auto readers = [&](const std::string& t) {
      std::vector<size_t> r;
      for (size_t j = 0; j < ops_.size(); ++j) {
        const OpSpec& o = ops_[j];
        bool reads = o.in0 == t || (o.type != OpType::Conv && o.in1 == t);
        for (const auto& a : o.adds) reads = reads || a == t;
        if (reads) r.push_back(j);
      }
      return r;
    };
    for (size_t i = 0; i < ops_.size() && !changed; ++i) {
      const OpSpec& add = ops_[i];
      if (add.type != OpType::Add || add.in0 == add.in1) continue;
      auto pa = producer.find(add.in0), pb = producer.find(add.in1);
      if (pa == producer.end() || pb == producer.end()) continue;
      const bool a_main = pa->second >= pb->second;
      const size_t main = a_main ? pa->second : pb->second;
      const std::string& main_out = a_main ? add.in0 : add.in1;
      const std::string& other = a_main ? add.in1 : add.in0;
      OpSpec& conv = ops_[main];
      if (conv.type != OpType::Conv || conv.out != main_out || conv.adds.size() >= 2 || conv.fuse_dts) continue;
      const auto r = readers(main_out);
      if (protected_out.count(main_out) || main_out == output_name_ || r.size() != 1 || r[0] != i) continue;
      conv.adds.push_back(other);
      conv.out = add.out;
      ops_.erase(ops_.begin() + static_cast<std::ptrdiff_t>(i));
      changed = true;
    }
  }

  // DepthToSpace fusion into a narrow producing conv (the upscaler tail): the conv
  // writes the rearranged (and clipped) result directly.
  for (size_t i = 0; i < ops_.size(); ++i) {
    if (ops_[i].type != OpType::DepthToSpace) continue;
    const std::string src = ops_[i].in0;
    size_t p = ops_.size();
    for (size_t j = 0; j < i; ++j)
      if (ops_[j].out == src) p = j;
    if (p == ops_.size() || ops_[p].type != OpType::Conv || ops_[p].fuse_dts) continue;
    const WeightSpec& ws = weights_[ops_[p].in1];
    if (ws.shape[0] > 16) continue;
    size_t readers = 0;
    for (const auto& o : ops_) {
      readers += (o.in0 == src) + (o.type != OpType::Conv && o.in1 == src);
      for (const auto& a : o.adds) readers += (a == src);
    }
    if (readers != 1 || protected_out.count(src) || src == output_name_) continue;
    OpSpec& conv = ops_[p];
    conv.fuse_dts = true;
    conv.blocksize = ops_[i].blocksize;
    conv.fuse_clip = ops_[i].fuse_clip;
    conv.clip_min = ops_[i].clip_min;
    conv.clip_max = ops_[i].clip_max;
    conv.out = ops_[i].out;
    ops_.erase(ops_.begin() + static_cast<std::ptrdiff_t>(i));
    --i;
  }

  // Clip fusion into a narrow producing conv without DepthToSpace (the chroma / dehalo
  // tails): the conv's per-element output path applies the bounds after its fp16 rounding,
  // activation and residual adds, which is the unfused graph's order.
  for (size_t i = 0; i < ops_.size(); ++i) {
    if (ops_[i].type != OpType::Clip) continue;
    const std::string src = ops_[i].in0;
    size_t p = ops_.size();
    for (size_t j = 0; j < i; ++j)
      if (ops_[j].out == src) p = j;
    if (p == ops_.size() || ops_[p].type != OpType::Conv || ops_[p].fuse_clip) continue;
    if (weights_[ops_[p].in1].shape[0] > 16) continue;
    size_t readers = 0;
    for (const auto& o : ops_) {
      readers += (o.in0 == src) + (o.type != OpType::Conv && o.in1 == src);
      for (const auto& a : o.adds) readers += (a == src);
    }
    if (readers != 1 || protected_out.count(src) || src == output_name_) continue;
    OpSpec& conv = ops_[p];
    conv.fuse_clip = true;
    conv.clip_min = ops_[i].clip_min;
    conv.clip_max = ops_[i].clip_max;
    conv.out = ops_[i].out;
    ops_.erase(ops_.begin() + static_cast<std::ptrdiff_t>(i));
    --i;
  }

  // Operand validation: elementwise ops read activations produced inside this graph,
  // never initializer constants or broadcasts (not implemented by the kernels).
  {
    std::unordered_set<std::string> produced;
    for (const auto& o : ops_) produced.insert(o.out);
    auto need = [&](const std::string& what, const std::string& name) {
      if (produced.count(name)) return true;
      error = what + " operand '" + name +
              "' is not an activation produced in this graph; initializer constants, graph inputs and "
              "broadcasting are not supported";
      return false;
    };
    for (const auto& o : ops_) {
      if (o.type == OpType::Mul || o.type == OpType::Add) {
        if (!need(OpTypeName(o.type), o.in0) || !need(OpTypeName(o.type), o.in1)) return false;
      } else if (o.type == OpType::Conv) {
        for (const auto& a : o.adds)
          if (!need("fused residual Add", a)) return false;
      }
    }
  }
  conv_widx_.assign(ops_.size(), -1);
  int nconv = 0;
  for (size_t i = 0; i < ops_.size(); ++i)
    if (ops_[i].type == OpType::Conv) conv_widx_[i] = nconv++;
  return true;
}

std::string Engine::Describe() const {
  std::ostringstream os;
  os << "input " << input_name_ << (input_is_fp32_ ? " fp32" : " fp16") << "\n";
  for (const auto& o : ops_) {
    os << OpTypeName(o.type) << " " << o.in0;
    if (o.type == OpType::Conv) {
      const auto& w = weights_.at(o.in1);
      os << " w=" << w.shape[1] << "->" << w.shape[0];
      if (o.act == kActRelu) os << " +relu";
      if (o.act == kActSilu) os << " +silu";
      for (const auto& a : o.adds) os << " +add(" << a << ")";
      if (o.fuse_dts) os << " +dts" << o.blocksize;
    } else if (!o.in1.empty()) {
      os << " " << o.in1;
    }
    if (o.type == OpType::DepthToSpace) os << " b=" << o.blocksize;
    if (o.fuse_clip || o.type == OpType::Clip) os << " clip[" << o.clip_min << "," << o.clip_max << "]";
    os << " -> " << o.out << "\n";
  }
  os << "output " << output_name_ << (output_is_fp32_ ? " fp32" : " fp16") << "\n";
  return os.str();
}

int Engine::InputChannels() const {
  for (const auto& o : ops_)
    if (o.type == OpType::Conv) return static_cast<int>(weights_.at(o.in1).shape[1]);
  return 1;
}

int Engine::OutputChannels() const {
  for (auto it = ops_.rbegin(); it != ops_.rend(); ++it)
    if (it->type == OpType::Conv) return static_cast<int>(weights_.at(it->in1).shape[0]);
  return 1;
}

// ---------------------------------------------------------------------------
// Shapes (internal tensors are NHWC)
// ---------------------------------------------------------------------------
bool Engine::PropagateShapes(const std::vector<int64_t>& s4,
                             std::unordered_map<std::string, std::vector<int64_t>>& shapes) const {
  if (s4.size() != 4 || s4[0] != 1) return false;  // no batch dimension in the kernels
  if (s4[1] <= 0 || s4[2] <= 0 || s4[3] <= 0) return false;
  shapes.clear();
  shapes[input_name_] = {s4[0], s4[2], s4[3], s4[1]};
  for (const auto& op : ops_) {
    auto it = shapes.find(op.in0);
    if (it == shapes.end()) return false;
    const std::vector<int64_t> s = it->second;
    std::vector<int64_t> o;
    switch (op.type) {
      case OpType::Conv: {
        const auto& w = weights_.at(op.in1);
        if (w.shape[1] != s[3]) return false;  // channel agreement
        o = {s[0], s[1], s[2], w.shape[0]};
        for (const auto& a : op.adds) {
          auto ai = shapes.find(a);
          if (ai == shapes.end() || ai->second != o) return false;
        }
        if (op.fuse_dts) {
          const int64_t b = op.blocksize;
          if (o[3] % (b * b)) return false;
          o = {o[0], o[1] * b, o[2] * b, o[3] / (b * b)};
        }
        break;
      }
      case OpType::Sigmoid:
      case OpType::Relu:
      case OpType::Clip:
        o = s;
        break;
      case OpType::Mul:
      case OpType::Add: {
        auto r = shapes.find(op.in1);
        if (r == shapes.end() || r->second != s) return false;  // same-shape elementwise only
        o = s;
        break;
      }
      case OpType::DepthToSpace: {
        const int64_t b = op.blocksize;
        if (b < 1 || s[3] % (b * b)) return false;
        o = {s[0], s[1] * b, s[2] * b, s[3] / (b * b)};
        break;
      }
    }
    shapes[op.out] = o;
  }
  return shapes.count(output_name_) != 0;
}

bool Engine::GetOutputShape(const std::vector<int64_t>& in, std::vector<int64_t>& out) const {
  std::unordered_map<std::string, std::vector<int64_t>> shapes;
  if (!PropagateShapes(in, shapes)) return false;
  const auto& o = shapes.at(output_name_);
  out = {o[0], o[3], o[1], o[2]};
  return true;
}

// ---------------------------------------------------------------------------
// Device state
// ---------------------------------------------------------------------------
void* Engine::BufPtr(int idx) const { return idx >= 0 ? bufs_[idx] : nullptr; }

void Engine::DestroyShapeState() {
  cudaSetDevice(device_id_);
  if (graph_exec_) cudaGraphExecDestroy(graph_exec_);
  graph_exec_ = nullptr;
  for (void* p : bufs_)
    if (p) cudaFree(p);
  bufs_.clear();
  buf_bytes_.clear();
  tensor_buf_.clear();
  dev_ops_.clear();
  if (in_boundary_ && !in_alias_) cudaFree(in_boundary_);
  if (out_boundary_ && !out_alias_) cudaFree(out_boundary_);
  in_boundary_ = out_boundary_ = nullptr;
  in_alias_ = out_alias_ = false;
  if (in_staging_) cudaFreeHost(in_staging_);
  if (out_staging_) cudaFreeHost(out_staging_);
  in_staging_ = out_staging_ = nullptr;
  for (cudaEvent_t e : prof_events_) cudaEventDestroy(e);
  prof_events_.clear();
  for (cudaEvent_t e : tevents_) cudaEventDestroy(e);
  tevents_.clear();
  t_max_frames_ = t_frames_ = 0;
  built_ = false;
  built_shape_.clear();
}

void Engine::DestroyAll() {
  DestroyShapeState();
  FreeWeights();
  if (status_) cudaFree(status_);
  status_ = nullptr;
  if (stream_) cudaStreamDestroy(stream_);
  stream_ = nullptr;
}

void Engine::FreeWeights() {
  for (auto& cw : conv_weights_) {
    conv_tc_free(&cw.tcw);
    simt_conv_free(&cw.sw);
    wino_free(&cw.ww);
  }
  conv_weights_.clear();
  weights_uploaded_ = false;
}

bool Engine::SetConvAlgo(int algo, std::string& error) {
  std::lock_guard<std::mutex> lock(mutex_);
  if (algo != 0 && algo != 1) {
    error = "conv algorithm must be 0 (direct) or 1 (winograd)";
    return false;
  }
  if (algo == conv_algo_) return true;
  if (!SetDevice(error)) return false;
  // Weights are packed per algorithm: drop the plan and the packed weights, rebuilt lazily.
  DestroyShapeState();
  FreeWeights();
  conv_algo_ = algo;
  return true;
}

bool Engine::UploadWeights(std::string& error) {
  if (weights_uploaded_) return true;
  conv_weights_.clear();
  for (size_t i = 0; i < ops_.size(); ++i) {
    const OpSpec& op = ops_[i];
    if (op.type != OpType::Conv) continue;
    const WeightSpec& ws = weights_.at(op.in1);
    const int M = static_cast<int>(ws.shape[0]), C = static_cast<int>(ws.shape[1]);
    std::vector<uint16_t> w16(static_cast<size_t>(M) * C * 9);
    for (size_t k = 0; k < w16.size(); ++k) w16[k] = WeightHalf(ws, k);
    std::vector<float> bias(M, 0.f);
    if (!op.bias.empty()) {
      const WeightSpec& bs = weights_.at(op.bias);
      for (int m = 0; m < M; ++m) bias[m] = HalfToFloat(WeightHalf(bs, m));
    }
    ConvWeights cw;
    // Winograd only where its output form applies: a plain NHWC activation (not a fused
    // DepthToSpace / Clip tail).
    // The direct form's weights are always packed: it also runs a Winograd-eligible conv
    // whose output is the graph boundary (NCHW in the IO dtype).
    cw.wino = conv_algo_ == 1 && wino_supported(C, M) && !op.fuse_dts && !op.fuse_clip;
    cw.tc = conv_tc_supported(C, M, nullptr);
    cudaError_t e = cw.tc ? conv_tc_upload(w16.data(), bias.data(), C, M, &cw.tcw)
                          : simt_conv_upload(w16.data(), bias.data(), C, M, &cw.sw);
    if (e == cudaSuccess && cw.wino) e = wino_upload(w16.data(), bias.data(), C, M, &cw.ww);
    conv_weights_.push_back(cw);
    if (e != cudaSuccess) {
      error = std::string("cudaMalloc/cudaMemcpy of conv weights failed: ") + cudaGetErrorString(e);
      return false;
    }
  }
  weights_uploaded_ = true;
  return true;
}

bool Engine::EnsureBuilt(const std::vector<int64_t>& s4, std::string& error) {
  if (built_ && s4 == built_shape_) return true;
  if (!device_ready_) {
    error = "engine is not built";
    return false;
  }
  if (!SetDevice(error)) return false;
  if (s4.size() != 4) {
    error = "expected 4D input tensor";
    return false;
  }
  if (s4[0] != 1) {
    error = "batch size must be 1 (the kernels do not implement a batch dimension)";
    return false;
  }
  DestroyShapeState();
  std::unordered_map<std::string, std::vector<int64_t>> shapes;
  if (!PropagateShapes(s4, shapes)) {
    error = "shape propagation failed (unsupported convolution geometry, channel mismatch, or DepthToSpace "
            "block size)";
    return false;
  }
  if (!UploadWeights(error)) return false;
  auto fail = [&](const std::string& what, cudaError_t e) {
    error = what + " failed: " + cudaGetErrorString(e);
    (void)cudaGetLastError();
    DestroyShapeState();
    return false;
  };

  // Liveness-based buffer assignment: a buffer is reused by a later tensor once every
  // reader of its previous tensor has run.
  std::unordered_map<std::string, int> last_use;
  for (size_t i = 0; i < ops_.size(); ++i) {
    const OpSpec& o = ops_[i];
    last_use[o.in0] = static_cast<int>(i);
    if (o.type != OpType::Conv && !o.in1.empty()) last_use[o.in1] = static_cast<int>(i);
    for (const auto& a : o.adds) last_use[a] = static_cast<int>(i);
  }
  last_use[output_name_] = static_cast<int>(ops_.size()) + 1;
  std::vector<int> free_after(0);
  std::vector<int> buf_free_at;  // op index after which the buffer's current tensor is dead
  auto alloc = [&](const std::string& name, int producer) -> int {
    auto it = tensor_buf_.find(name);
    if (it != tensor_buf_.end()) return it->second;
    const size_t bytes = static_cast<size_t>(Numel(shapes.at(name))) * 2;
    int best = -1;
    for (size_t b = 0; b < bufs_.size(); ++b) {
      if (buf_free_at[b] < producer && buf_bytes_[b] >= bytes && (best < 0 || buf_bytes_[b] < buf_bytes_[best]))
        best = static_cast<int>(b);
    }
    if (best < 0) {
      void* p = nullptr;
      cudaError_t e = cudaMalloc(&p, bytes);
      if (e != cudaSuccess) {
        error = "cudaMalloc of " + std::to_string(bytes) + " bytes for tensor '" + name +
                "' failed: " + cudaGetErrorString(e);
        (void)cudaGetLastError();
        return -1;
      }
      bufs_.push_back(p);
      buf_bytes_.push_back(bytes);
      buf_free_at.push_back(0);
      best = static_cast<int>(bufs_.size()) - 1;
    }
    auto lu = last_use.find(name);
    buf_free_at[best] = lu == last_use.end() ? producer : lu->second;
    tensor_buf_[name] = best;
    return best;
  };

  if (alloc(input_name_, -1) < 0) {
    DestroyShapeState();
    return false;
  }

  const auto& in_nhwc = shapes.at(input_name_);
  const auto& out_nhwc = shapes.at(output_name_);
  const int inC = static_cast<int>(in_nhwc[3]), inH = static_cast<int>(in_nhwc[1]), inW = static_cast<int>(in_nhwc[2]);
  const int outC = static_cast<int>(out_nhwc[3]), outH = static_cast<int>(out_nhwc[1]),
            outW = static_cast<int>(out_nhwc[2]);
  in_bytes_ = static_cast<size_t>(Numel(in_nhwc)) * (input_is_fp32_ ? 4 : 2);
  out_bytes_ = static_cast<size_t>(Numel(out_nhwc)) * (output_is_fp32_ ? 4 : 2);

  // Which op produces the graph output, and can it write the boundary layout itself?
  int out_op = -1;
  for (size_t i = 0; i < ops_.size(); ++i)
    if (ops_[i].out == output_name_) out_op = static_cast<int>(i);
  const bool out_needs_convert = output_is_fp32_ || outC > 1;
  bool out_direct = false;
  if (out_op >= 0 && out_needs_convert) {
    const OpSpec& o = ops_[out_op];
    if (o.type == OpType::DepthToSpace || o.type == OpType::Conv) out_direct = true;
  }

  for (size_t i = 0; i < ops_.size(); ++i) {
    const OpSpec& o = ops_[i];
    const int pi = static_cast<int>(i);
    const bool direct_here = out_direct && pi == out_op;
    // In place: a conv whose last residual operand dies at this op writes its result over
    // that operand (the tensor-core conv then adds the operand in L2 with reduce-add tile
    // stores; the other conv kernels read each residual element before writing it). Not
    // for the graph input, nor when the operand is also the conv's input or its first
    // residual.
    if (!direct_here && o.type == OpType::Conv && !o.adds.empty() && !o.fuse_dts && !o.fuse_clip &&
        !tensor_buf_.count(o.out)) {
      const std::string& r = o.adds.back();
      const auto rb = tensor_buf_.find(r);
      if (r != input_name_ && r != o.in0 && (o.adds.size() == 1 || o.adds[0] != r) && last_use.at(r) == pi &&
          rb != tensor_buf_.end() && buf_bytes_[rb->second] >= static_cast<size_t>(Numel(shapes.at(o.out))) * 2) {
        tensor_buf_[o.out] = rb->second;
        auto lu = last_use.find(o.out);
        buf_free_at[rb->second] = lu == last_use.end() ? pi : lu->second;
      }
    }
    if (!direct_here && alloc(o.out, pi) < 0) {
      DestroyShapeState();
      return false;
    }
  }

  // Boundary buffers.
  {
    cudaError_t e;
    if (input_is_fp32_ || inC > 1) {
      e = cudaMalloc(&in_boundary_, in_bytes_);
      if (e != cudaSuccess) return fail("cudaMalloc of the input boundary buffer", e);
    } else {
      in_boundary_ = bufs_[tensor_buf_.at(input_name_)];
      in_alias_ = true;
    }
    if (out_needs_convert) {
      e = cudaMalloc(&out_boundary_, out_bytes_);
      if (e != cudaSuccess) return fail("cudaMalloc of the output boundary buffer", e);
    } else {
      out_boundary_ = bufs_[tensor_buf_.at(output_name_)];
      out_alias_ = true;
    }
    e = cudaMallocHost(&in_staging_, in_bytes_);
    if (e != cudaSuccess) return fail("cudaMallocHost of input staging", e);
    e = cudaMallocHost(&out_staging_, out_bytes_);
    if (e != cudaSuccess) return fail("cudaMallocHost of output staging", e);
  }

  // Device op list.
  if (input_is_fp32_ || inC > 1) {
    DevOp d;
    d.kind = 5;
    d.C = inC;
    d.H = inH;
    d.W = inW;
    d.in_boundary = true;
    d.out_buf = tensor_buf_.at(input_name_);
    d.info.kind = "io";
    d.info.label = "input NCHW->NHWC";
    d.info.bytes = static_cast<double>(in_bytes_) + static_cast<double>(Numel(in_nhwc)) * 2;
    dev_ops_.push_back(d);
  }
  for (size_t i = 0; i < ops_.size(); ++i) {
    const OpSpec& o = ops_[i];
    const auto& is = shapes.at(o.in0);
    DevOp d;
    d.type = o.type;
    d.H = static_cast<int>(is[1]);
    d.W = static_cast<int>(is[2]);
    d.C = static_cast<int>(is[3]);
    d.in_buf = tensor_buf_.at(o.in0);
    const bool direct_here = out_direct && static_cast<int>(i) == out_op;
    d.out_boundary = direct_here;
    d.out_buf = direct_here ? -1 : tensor_buf_.at(o.out);
    const double P = static_cast<double>(d.H) * d.W;
    std::ostringstream lab;
    lab << OpTypeName(o.type) << " " << d.H << "x" << d.W;
    switch (o.type) {
      case OpType::Conv: {
        d.widx = conv_widx_[i];
        const ConvWeights& cw = conv_weights_[d.widx];
        d.M = static_cast<int>(weights_.at(o.in1).shape[0]);
        d.act = o.act;
        for (size_t k = 0; k < o.adds.size(); ++k) d.add_buf[k] = tensor_buf_.at(o.adds[k]);
        lab << " " << d.C << "->" << d.M << (o.act == kActRelu ? " relu" : (o.act == kActSilu ? " silu" : ""))
            << (o.adds.empty() ? "" : (o.adds.size() == 1 ? " +add" : " +add+add"))
            << (!o.adds.empty() && d.out_buf >= 0 && d.out_buf == d.add_buf[o.adds.size() - 1] ? " in place" : "")
            << (o.fuse_dts ? " +dts" : "");
        d.info.flops = 2.0 * 9.0 * d.C * d.M * P;
        d.info.bytes = 2.0 * P * d.C + 2.0 * P * d.M * (1.0 + o.adds.size()) + 2.0 * (9.0 * d.C * d.M + d.M);
        // Output form shared by both conv kernels: fused DepthToSpace / clip, and the
        // graph-boundary layout (NCHW, model dtype) when this op produces the output.
        d.sout.dts_b = o.fuse_dts ? o.blocksize : 1;
        d.sout.clip = o.fuse_clip ? 1 : 0;
        d.sout.clip_lo = o.clip_min;
        d.sout.clip_hi = o.clip_max;
        if (direct_here) {
          d.sout.nchw = 1;
          d.sout.fp32 = output_is_fp32_ ? 1 : 0;
        }
        if (cw.wino && !direct_here) {
          d.kind = 7;
          d.info.kind = "conv_wino";
          std::string perr;
          if (!wino_plan(&cw.ww, static_cast<const __half*>(bufs_[d.in_buf]), d.H, d.W,
                         static_cast<__half*>(bufs_[d.out_buf]), num_sms_, &d.wp, &perr)) {
            error = "conv plan failed: " + perr;
            DestroyShapeState();
            return false;
          }
        } else if (cw.tc) {
          d.kind = 0;
          d.info.kind = "conv_tc";
          ConvTcOut to;
          to.ptr = direct_here ? out_boundary_ : bufs_[d.out_buf];
          const bool plain = !o.fuse_dts && !o.fuse_clip && !direct_here && d.M % 16 == 0;
          to.mode = plain ? 0 : 1;
          to.dts_b = d.sout.dts_b;
          to.nchw = d.sout.nchw;
          to.fp32 = d.sout.fp32;
          to.clip = d.sout.clip;
          to.clip_lo = d.sout.clip_lo;
          to.clip_hi = d.sout.clip_hi;
          to.adds = (d.add_buf[0] >= 0 ? 1 : 0) + (d.add_buf[1] >= 0 ? 1 : 0);
          std::string perr;
          if (!conv_tc_plan(&cw.tcw, static_cast<const __half*>(bufs_[d.in_buf]), d.H, d.W, to, num_sms_, &d.tc,
                            &perr)) {
            error = "conv plan failed: " + perr;
            DestroyShapeState();
            return false;
          }
        } else {
          d.kind = 1;
          d.info.kind = "conv_simt";
        }
        break;
      }
      case OpType::Sigmoid:
      case OpType::Relu:
      case OpType::Clip:
        d.kind = 2;
        d.numel = static_cast<size_t>(Numel(is));
        d.subop = o.type == OpType::Sigmoid ? kSigmoid : (o.type == OpType::Relu ? kRelu : kClip);
        d.lo = o.clip_min;
        d.hi = o.clip_max;
        d.info.kind = "unary";
        d.info.bytes = 4.0 * d.numel;
        break;
      case OpType::Mul:
      case OpType::Add:
        d.kind = 3;
        d.numel = static_cast<size_t>(Numel(is));
        d.in1_buf = tensor_buf_.at(o.in1);
        d.subop = o.type == OpType::Mul ? kMul : kAdd;
        d.info.kind = "binary";
        d.info.bytes = 6.0 * d.numel;
        break;
      case OpType::DepthToSpace:
        d.kind = 4;
        d.sout.dts_b = o.blocksize;
        d.sout.clip = o.fuse_clip ? 1 : 0;
        d.sout.clip_lo = o.clip_min;
        d.sout.clip_hi = o.clip_max;
        if (direct_here) {
          d.sout.nchw = 1;
          d.sout.fp32 = output_is_fp32_ ? 1 : 0;
        }
        d.info.kind = "dts";
        d.info.bytes = 4.0 * static_cast<double>(Numel(is));
        break;
    }
    d.info.label = lab.str();
    dev_ops_.push_back(d);
  }
  if (out_needs_convert && !out_direct) {
    DevOp d;
    d.kind = 6;
    d.C = outC;
    d.H = outH;
    d.W = outW;
    d.in_buf = tensor_buf_.at(output_name_);
    d.out_boundary = true;
    d.info.kind = "io";
    d.info.label = "output NHWC->NCHW";
    d.info.bytes = static_cast<double>(out_bytes_) + static_cast<double>(Numel(out_nhwc)) * 2;
    dev_ops_.push_back(d);
  }
  if (prof_) {
    prof_events_.resize(dev_ops_.size() + 1);
    for (auto& ev : prof_events_) {
      cudaError_t e = cudaEventCreate(&ev);
      if (e != cudaSuccess) return fail("cudaEventCreate", e);
    }
  }
  built_ = true;
  built_shape_ = s4;
  return true;
}

// ---------------------------------------------------------------------------
// Execution
// ---------------------------------------------------------------------------
cudaError_t Engine::LaunchOp(size_t i, cudaStream_t s) {
  const DevOp& d = dev_ops_[i];
  cudaError_t e = cudaSuccess;
  const __half* in = d.in_boundary ? nullptr : static_cast<const __half*>(BufPtr(d.in_buf));
  void* out = d.out_boundary ? out_boundary_ : BufPtr(d.out_buf);
  switch (d.kind) {
    case 0:
      e = conv_tc_launch(d.tc, static_cast<const __half*>(BufPtr(d.add_buf[0])),
                         static_cast<const __half*>(BufPtr(d.add_buf[1])), d.act, status_, s);
      break;
    case 1: {
      SimtOut so = d.sout;
      so.ptr = out;
      e = simt_conv_launch(conv_weights_[d.widx].sw, in, d.H, d.W, static_cast<const __half*>(BufPtr(d.add_buf[0])),
                           static_cast<const __half*>(BufPtr(d.add_buf[1])), d.act, so, s);
      break;
    }
    case 2:
      e = unary_launch(in, static_cast<__half*>(out), d.numel, d.subop, d.lo, d.hi, s);
      break;
    case 3:
      e = binary_launch(in, static_cast<const __half*>(BufPtr(d.in1_buf)), static_cast<__half*>(out), d.numel,
                        d.subop, s);
      break;
    case 4: {
      SimtOut so = d.sout;
      so.ptr = out;
      e = dts_launch(in, d.H, d.W, d.C, so, s);
      break;
    }
    case 5:
      e = nchw_to_nhwc_launch(in_boundary_, input_is_fp32_ ? 1 : 0, static_cast<__half*>(out), d.C, d.H, d.W, s);
      break;
    case 6:
      e = nhwc_to_nchw_launch(in, out_boundary_, output_is_fp32_ ? 1 : 0, d.C, d.H, d.W, s);
      break;
    case 7:
      e = wino_launch(d.wp, static_cast<const __half*>(BufPtr(d.add_buf[0])),
                      static_cast<const __half*>(BufPtr(d.add_buf[1])), d.act, status_, s);
      break;
  }
  return e;
}

bool Engine::EnqueueOps(int begin, int end, std::string& error) {
  std::lock_guard<std::mutex> lock(mutex_);
  if (!built_) {
    error = "engine is not prepared for a shape";
    return false;
  }
  if (begin < 0 || end > static_cast<int>(dev_ops_.size()) || begin > end) {
    error = "op range [" + std::to_string(begin) + ", " + std::to_string(end) + ") outside the plan's " +
            std::to_string(dev_ops_.size()) + " ops";
    return false;
  }
  if (!SetDevice(error)) return false;
  for (int i = begin; i < end; ++i) {
    const cudaError_t e = LaunchOp(static_cast<size_t>(i), stream_);
    if (e != cudaSuccess) {
      error = "kernel launch for op " + std::to_string(i) + " (" + dev_ops_[i].info.label + ") failed: " +
              cudaGetErrorString(e);
      (void)cudaGetLastError();
      return false;
    }
  }
  return true;
}

bool Engine::OpOutput(int i, void** ptr, int* rows, size_t* row_bytes, bool* boundary) const {
  std::lock_guard<std::mutex> lock(mutex_);
  if (!built_ || i < 0 || i >= static_cast<int>(dev_ops_.size())) return false;
  const DevOp& d = dev_ops_[i];
  *boundary = d.out_boundary;
  *ptr = d.out_boundary ? out_boundary_ : BufPtr(d.out_buf);
  const int ch = (d.kind == 0 || d.kind == 1 || d.kind == 7) ? d.M : d.C;  // conv outputs M channels
  *rows = d.H;
  *row_bytes = static_cast<size_t>(d.W) * static_cast<size_t>(ch) * sizeof(__half);
  return true;
}

bool Engine::LaunchFrame(bool with_events, std::string& error) {
  cudaStream_t s = stream_;
  auto ev = [&](size_t k) -> cudaError_t {
    if (!with_events) return cudaSuccess;
    const size_t base = static_cast<size_t>(t_frames_) * (dev_ops_.size() + 1);
    return cudaEventRecord(tevents_[base + k], s);
  };
  if (prof_ && !prof_events_.empty()) cudaEventRecord(prof_events_[0], s);
  if (ev(0) != cudaSuccess) {
    error = "cudaEventRecord failed";
    return false;
  }
  for (size_t i = 0; i < dev_ops_.size(); ++i) {
    const DevOp& d = dev_ops_[i];
    cudaError_t e = LaunchOp(i, s);
    if (e != cudaSuccess) {
      error = "kernel launch for op " + std::to_string(i) + " (" + d.info.label + ") failed: " + cudaGetErrorString(e);
      (void)cudaGetLastError();
      return false;
    }
    if (prof_ && !prof_events_.empty()) cudaEventRecord(prof_events_[i + 1], s);
    if (ev(i + 1) != cudaSuccess) {
      error = "cudaEventRecord failed";
      return false;
    }
    if (sync_each_) {
      e = cudaStreamSynchronize(s);
      if (e != cudaSuccess) {
        error = "op " + std::to_string(i) + " (" + d.info.label + ") failed: " + cudaGetErrorString(e);
        return false;
      }
    }
  }
  if (with_events) ++t_frames_;
  return true;
}

bool Engine::CheckStatus(std::string& error) {
  uint32_t st = 0;
  cudaError_t e = cudaMemcpy(&st, status_, sizeof(st), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) {
    error = std::string("status read failed: ") + cudaGetErrorString(e);
    return false;
  }
  if (st != 0) {
    cudaMemset(status_, 0, sizeof(uint32_t));
    error = "tensor-core conv kernel reported a timed-out pipeline wait (status " + std::to_string(st) + ")";
    return false;
  }
  return true;
}

bool Engine::Enqueue(std::string& error) {
  std::lock_guard<std::mutex> lock(mutex_);
  if (!built_) {
    error = "engine is not prepared for a shape";
    return false;
  }
  if (!SetDevice(error)) return false;
  if (t_max_frames_ > 0) {
    if (t_frames_ >= t_max_frames_) {
      error = "timing event budget exhausted";
      return false;
    }
    return LaunchFrame(true, error);
  }
  if (no_graph_) return LaunchFrame(false, error);
  if (!graph_exec_) {
    // Capture the frame's launch sequence once per built plan.
    cudaGraph_t graph = nullptr;
    cudaError_t e = cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) {
      error = std::string("cudaStreamBeginCapture failed: ") + cudaGetErrorString(e);
      return false;
    }
    std::string lerr;
    const bool ok = LaunchFrame(false, lerr);
    e = cudaStreamEndCapture(stream_, &graph);
    if (!ok || e != cudaSuccess) {
      if (graph) cudaGraphDestroy(graph);
      error = ok ? std::string("cudaStreamEndCapture failed: ") + cudaGetErrorString(e) : lerr;
      (void)cudaGetLastError();
      return false;
    }
    e = cudaGraphInstantiate(&graph_exec_, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) {
      graph_exec_ = nullptr;
      error = std::string("cudaGraphInstantiate failed: ") + cudaGetErrorString(e);
      return false;
    }
  }
  cudaError_t e = cudaGraphLaunch(graph_exec_, stream_);
  if (e != cudaSuccess) {
    error = std::string("cudaGraphLaunch failed: ") + cudaGetErrorString(e);
    return false;
  }
  return true;
}

bool Engine::Synchronize(std::string& error) {
  if (!SetDevice(error)) return false;
  cudaError_t e = cudaStreamSynchronize(stream_);
  if (e != cudaSuccess) {
    error = std::string("stream synchronize failed: ") + cudaGetErrorString(e);
    return false;
  }
  return CheckStatus(error);
}

bool Engine::Prepare(const std::vector<int64_t>& s4, void** in_dev, void** out_dev, size_t* in_bytes,
                     size_t* out_bytes, std::string& error) {
  std::lock_guard<std::mutex> lock(mutex_);
  (void)cudaGetLastError();
  if (!SetDevice(error)) return false;
  if (!EnsureBuilt(s4, error)) return false;
  if (in_dev) *in_dev = in_boundary_;
  if (out_dev) *out_dev = out_boundary_;
  if (in_bytes) *in_bytes = in_bytes_;
  if (out_bytes) *out_bytes = out_bytes_;
  return true;
}

bool Engine::TimingStart(int max_frames, std::string& error) {
  std::lock_guard<std::mutex> lock(mutex_);
  if (!built_) {
    error = "engine is not prepared for a shape";
    return false;
  }
  for (cudaEvent_t e : tevents_) cudaEventDestroy(e);
  tevents_.assign(static_cast<size_t>(max_frames) * (dev_ops_.size() + 1), nullptr);
  for (auto& ev : tevents_) {
    cudaError_t e = cudaEventCreate(&ev);
    if (e != cudaSuccess) {
      error = std::string("cudaEventCreate failed: ") + cudaGetErrorString(e);
      return false;
    }
  }
  t_max_frames_ = max_frames;
  t_frames_ = 0;
  return true;
}

bool Engine::TimingRead(std::vector<double>* op_ms, double* span_ms, int* frames, std::string& error) {
  std::lock_guard<std::mutex> lock(mutex_);
  if (!SetDevice(error)) return false;
  cudaError_t e = cudaStreamSynchronize(stream_);
  if (e != cudaSuccess) {
    error = std::string("stream synchronize failed: ") + cudaGetErrorString(e);
    return false;
  }
  const size_t nops = dev_ops_.size();
  op_ms->assign(nops, 0.0);
  *span_ms = 0.0;
  *frames = t_frames_;
  for (int f = 0; f < t_frames_; ++f) {
    const size_t base = static_cast<size_t>(f) * (nops + 1);
    for (size_t i = 0; i < nops; ++i) {
      float ms = 0.f;
      cudaEventElapsedTime(&ms, tevents_[base + i], tevents_[base + i + 1]);
      (*op_ms)[i] += ms;
    }
  }
  if (t_frames_ > 0) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, tevents_[0], tevents_[static_cast<size_t>(t_frames_ - 1) * (nops + 1) + nops]);
    *span_ms = ms;
  }
  for (cudaEvent_t ev : tevents_) cudaEventDestroy(ev);
  tevents_.clear();
  t_max_frames_ = 0;
  t_frames_ = 0;
  return CheckStatus(error);
}

std::vector<Engine::OpInfo> Engine::DeviceOps() const {
  std::vector<OpInfo> v;
  for (const auto& d : dev_ops_) v.push_back(d.info);
  return v;
}

bool Engine::Run(const void* input, const std::vector<int64_t>& s4, void* output, std::string& error) {
  std::lock_guard<std::mutex> lock(mutex_);
  const uint64_t no = ++frame_no_;
  if (trace_) std::fprintf(stderr, "[run] enter #%llu in=%p\n", static_cast<unsigned long long>(no), input);
  (void)cudaGetLastError();  // an earlier failure on this thread must not be blamed on this frame
  if (!SetDevice(error)) return false;
  if (!EnsureBuilt(s4, error)) return false;
  if (!input || !output) {
    error = "null input or output buffer";
    return false;
  }
  auto run_fail = [&](const char* what, cudaError_t e) {
    error = std::string(what) + " failed: " + cudaGetErrorString(e);
    (void)cudaGetLastError();
    return false;
  };
  auto pinned = [](const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
      (void)cudaGetLastError();
      return false;
    }
    return a.type == cudaMemoryTypeHost;
  };
  if (poison_) {
    for (size_t b = 0; b < bufs_.size(); ++b) {
      cudaError_t e = cudaMemsetAsync(bufs_[b], 0x7E, buf_bytes_[b], stream_);  // fp16 NaN pattern
      if (e != cudaSuccess) return run_fail("poison memset", e);
    }
  }
  const void* src = input;
  if (!pinned(input)) {
    std::memcpy(in_staging_, input, in_bytes_);
    src = in_staging_;
  }
  cudaError_t e = cudaMemcpyAsync(in_boundary_, src, in_bytes_, cudaMemcpyHostToDevice, stream_);
  if (e != cudaSuccess) return run_fail("input upload", e);
  // Enqueue without re-locking: inline the graph / direct launch.
  if (no_graph_ || t_max_frames_ > 0) {
    if (!LaunchFrame(false, error)) return false;
  } else {
    if (!graph_exec_) {
      cudaGraph_t graph = nullptr;
      e = cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal);
      if (e != cudaSuccess) return run_fail("cudaStreamBeginCapture", e);
      std::string lerr;
      const bool ok = LaunchFrame(false, lerr);
      e = cudaStreamEndCapture(stream_, &graph);
      if (!ok) {
        if (graph) cudaGraphDestroy(graph);
        error = lerr;
        return false;
      }
      if (e != cudaSuccess) return run_fail("cudaStreamEndCapture", e);
      e = cudaGraphInstantiate(&graph_exec_, graph, 0);
      cudaGraphDestroy(graph);
      if (e != cudaSuccess) {
        graph_exec_ = nullptr;
        return run_fail("cudaGraphInstantiate", e);
      }
    }
    e = cudaGraphLaunch(graph_exec_, stream_);
    if (e != cudaSuccess) return run_fail("cudaGraphLaunch", e);
  }
  void* dst = pinned(output) ? output : out_staging_;
  e = cudaMemcpyAsync(dst, out_boundary_, out_bytes_, cudaMemcpyDeviceToHost, stream_);
  if (e != cudaSuccess) return run_fail("output download", e);
  e = cudaStreamSynchronize(stream_);
  if (e != cudaSuccess) return run_fail("stream synchronize", e);
  if (!CheckStatus(error)) return false;
  if (prof_ && !prof_events_.empty()) {
    const bool report = frame_no_ <= 3 || frame_no_ % 128 == 0;
    if (report) {
      std::fprintf(stderr, "[vship-prof] frame %llu\n", static_cast<unsigned long long>(frame_no_));
      for (size_t i = 0; i < dev_ops_.size(); ++i) {
        float ms = 0.f;
        cudaEventElapsedTime(&ms, prof_events_[i], prof_events_[i + 1]);
        std::fprintf(stderr, "[vship-prof] op%-2zu type=%d %8.3f ms  %s\n", i, dev_ops_[i].kind, ms,
                     dev_ops_[i].info.label.c_str());
      }
    }
  }
  if (dst != output) std::memcpy(output, out_staging_, out_bytes_);
  if (trace_) std::fprintf(stderr, "[run] done    #%llu out=%p\n", static_cast<unsigned long long>(no), output);
  return true;
}

}  // namespace ah
