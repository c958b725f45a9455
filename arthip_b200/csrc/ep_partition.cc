// Partition rules of the ONNX Runtime execution provider (see ep_partition.h).
#include "ep_partition.h"

#include <atomic>
#include <unordered_set>

namespace ah {
namespace ep {

namespace {

bool IsDefaultDomain(const std::string& d) { return d.empty() || d == "ai.onnx"; }

std::unordered_set<std::string> InitializerNames(const onnx::Graph& g) {
  std::unordered_set<std::string> s;
  for (const auto& t : g.initializers) s.insert(t.name);
  return s;
}

// Graph inputs that are not initializers (ORT's GraphViewer::GetInputs()).
std::unordered_set<std::string> ActivationInputs(const onnx::Graph& g) {
  const auto inits = InitializerNames(g);
  std::unordered_set<std::string> s;
  for (const auto& v : g.inputs)
    if (!inits.count(v.name)) s.insert(v.name);
  return s;
}

std::unordered_set<std::string> OutputNames(const onnx::Graph& g) {
  std::unordered_set<std::string> s;
  for (const auto& v : g.outputs) s.insert(v.name);
  return s;
}

const onnx::Tensor* FindInitializer(const onnx::Graph& g, const std::string& name) {
  for (const auto& t : g.initializers)
    if (t.name == name) return &t;
  return nullptr;
}

int TypeOf(const std::unordered_map<std::string, int>& types, const std::string& name) {
  auto it = types.find(name);
  return it == types.end() ? 0 : it->second;
}

}  // namespace

std::unordered_map<std::string, int> InferElemTypes(const onnx::Graph& g) {
  std::unordered_map<std::string, int> t;
  for (const auto& v : g.inputs) t[v.name] = v.elem_type;
  for (const auto& i : g.initializers) t[i.name] = i.data_type;
  for (const auto& n : g.nodes) {
    int ty = 0;
    if (n.op_type == "Cast") {
      if (const auto* a = n.attr("to")) ty = static_cast<int>(a->i);
    } else if (!n.inputs.empty() && !n.inputs[0].empty()) {
      ty = TypeOf(t, n.inputs[0]);
    }
    for (const auto& o : n.outputs)
      if (!o.empty()) t[o] = ty;
  }
  // Declared graph output types fill values the rule above could not type.
  for (const auto& v : g.outputs)
    if (TypeOf(t, v.name) == 0) t[v.name] = v.elem_type;
  return t;
}

bool IsNodeSupported(const onnx::Graph& g, int index, const std::unordered_map<std::string, int>& types) {
  if (index < 0 || index >= static_cast<int>(g.nodes.size())) return false;
  const onnx::Node& n = g.nodes[index];
  const std::string& op = n.op_type;
  if (op == "Cast") {
    // Only the boundary Casts, which the engine folds into its IO conversion: fp32 graph
    // input -> fp16, and fp16 -> fp32 graph output.
    if (n.inputs.empty() || n.outputs.empty() || n.inputs[0].empty() || n.outputs[0].empty()) return false;
    const int in_t = TypeOf(types, n.inputs[0]), out_t = TypeOf(types, n.outputs[0]);
    if (in_t == onnx::kFloat && out_t == onnx::kFloat16) return ActivationInputs(g).count(n.inputs[0]) != 0;
    if (in_t == onnx::kFloat16 && out_t == onnx::kFloat) return OutputNames(g).count(n.outputs[0]) != 0;
    return false;
  }
  if (op != "Conv" && op != "Sigmoid" && op != "Mul" && op != "Add" && op != "DepthToSpace" && op != "Clip" &&
      op != "Relu")
    return false;
  if (!IsDefaultDomain(n.domain)) return false;
  // Every value the node reads or writes is fp16 (missing optional inputs are skipped).
  for (const auto& v : n.inputs)
    if (!v.empty() && TypeOf(types, v) != onnx::kFloat16) return false;
  for (const auto& v : n.outputs)
    if (!v.empty() && TypeOf(types, v) != onnx::kFloat16) return false;

  if (op == "Conv") {
    if (const auto* a = n.attr("strides"); a && a->ints.size() >= 2 && (a->ints[0] != 1 || a->ints[1] != 1))
      return false;
    if (const auto* a = n.attr("dilations"); a && a->ints.size() >= 2 && (a->ints[0] != 1 || a->ints[1] != 1))
      return false;
    if (const auto* a = n.attr("group"); a && a->i != 1) return false;
    // Symmetric 1-padding on both axes only; ONNX pads are [top, left, bottom, right].
    bool pads_ok = false;
    if (const auto* a = n.attr("pads")) {
      if (a->ints.size() != 4 || a->ints[0] != 1 || a->ints[1] != 1 || a->ints[2] != 1 || a->ints[3] != 1)
        return false;
      pads_ok = true;
    }
    if (const auto* a = n.attr("auto_pad")) {
      if (a->s == "SAME_UPPER" || a->s == "SAME_LOWER") pads_ok = true;
      else if (a->s != "NOTSET") return false;  // VALID: no padding, which the kernels do not do
    }
    if (!pads_ok) return false;
    if (n.inputs.size() < 2) return false;
    const onnx::Tensor* w = FindInitializer(g, n.inputs[1]);
    if (!w || w->dims.size() != 4 || w->dims[2] != 3 || w->dims[3] != 3) return false;
  }
  if (op == "DepthToSpace") {
    if (const auto* a = n.attr("mode"); a && a->s != "DCR") return false;
    if (const auto* a = n.attr("blocksize"); a && a->i < 1) return false;
  }
  if (op == "Clip") {
    // Input-form bounds must be initializers: a dynamic bound cannot be evaluated here.
    for (size_t i = 1; i < n.inputs.size(); ++i)
      if (!n.inputs[i].empty() && !FindInitializer(g, n.inputs[i])) return false;
  }
  return true;
}

std::vector<Region> GetCapability(const onnx::Model& m, bool context_ok) {
  std::vector<Region> result;
  if (!context_ok) return result;
  const onnx::Graph& g = m.graph;
  const auto types = InferElemTypes(g);

  // Maximal runs of consecutive supported nodes.
  std::vector<std::vector<int>> runs;
  std::vector<int> cur;
  for (int i = 0; i < static_cast<int>(g.nodes.size()); ++i) {
    if (IsNodeSupported(g, i, types)) {
      cur.push_back(i);
    } else if (!cur.empty()) {
      runs.push_back(cur);
      cur.clear();
    }
  }
  if (!cur.empty()) runs.push_back(cur);

  static std::atomic<int> metadef_id{0};
  const auto graph_outputs = OutputNames(g);
  const auto inits = InitializerNames(g);
  std::unordered_map<std::string, int> total_consumers;
  for (const auto& n : g.nodes)
    for (const auto& v : n.inputs)
      if (!v.empty()) ++total_consumers[v];

  for (const auto& run : runs) {
    std::unordered_set<std::string> produced;
    std::unordered_map<std::string, int> inside;
    for (int i : run)
      for (const auto& v : g.nodes[i].outputs)
        if (!v.empty()) produced.insert(v);
    for (int i : run)
      for (const auto& v : g.nodes[i].inputs)
        if (!v.empty()) ++inside[v];
    Region r;
    r.nodes = run;
    std::unordered_set<std::string> seen_act, seen_const, seen_out;
    for (int i : run) {
      for (const auto& v : g.nodes[i].inputs) {
        if (v.empty() || produced.count(v)) continue;
        if (inits.count(v)) {
          if (seen_const.insert(v).second) r.constants.push_back(v);
        } else if (seen_act.insert(v).second) {
          r.activations.push_back(v);
        }
      }
      for (const auto& v : g.nodes[i].outputs) {
        if (v.empty()) continue;
        const int in_run = inside.count(v) ? inside.at(v) : 0;
        const int total = total_consumers.count(v) ? total_consumers.at(v) : 0;
        if ((total > in_run || graph_outputs.count(v)) && seen_out.insert(v).second) r.outputs.push_back(v);
      }
    }
    // The compiled engine reads one input and writes one output: other runs are left to
    // another provider rather than claimed and run with an input dropped.
    if (r.activations.size() != 1 || r.outputs.size() != 1) continue;
    r.name = "HipKernel_graph_" + std::to_string(metadef_id.fetch_add(1));
    result.push_back(std::move(r));
  }
  return result;
}

onnx::Model RegionModel(const onnx::Model& m, const Region& r) {
  const onnx::Graph& g = m.graph;
  const auto types = InferElemTypes(g);
  onnx::Model out;
  out.ir_version = m.ir_version;
  out.opset = m.opset;
  for (int i : r.nodes) out.graph.nodes.push_back(g.nodes[i]);
  auto value_info = [&](const std::string& name) {
    onnx::ValueInfo v;
    v.name = name;
    v.elem_type = TypeOf(types, name);
    for (const auto& d : g.inputs)
      if (d.name == name) v.dims = d.dims;
    for (const auto& d : g.outputs)
      if (d.name == name) v.dims = d.dims;
    return v;
  };
  for (const auto& a : r.activations) out.graph.inputs.push_back(value_info(a));
  for (const auto& o : r.outputs) out.graph.outputs.push_back(value_info(o));
  for (const auto& c : r.constants)
    if (const onnx::Tensor* t = FindInitializer(g, c)) out.graph.initializers.push_back(*t);
  return out;
}

}  // namespace ep
}  // namespace ah
