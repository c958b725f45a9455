// Partition rules of the ONNX Runtime execution provider, in the engine core (no ORT
// headers): which nodes the provider can run, the maximal node runs it claims, and the
// standalone model of a claimed run that the engine compiles.
//
// Follows HIPExecutionProvider::GetCapability / IsNodeSupported / Compile
// (src/onnxruntime-hip/hip_execution_provider.cc:22-161, 180-335, 337-406). ORT hands the
// provider a GraphViewer whose NodeArgs carry inferred types; here the model bytes are
// decoded and the element types of the values are inferred for the operators in scope
// (Cast: its `to`; every other operator: the type of its first input, which holds for all
// the elementwise / conv / layout operators the provider runs). Nodes are visited in the
// model's node order, which ONNX requires to be topological.
//
// Differences from the reference, on purpose:
//  * Relu is claimed as well (the engine fuses it; the reference has no Relu support);
//  * a claimed run compiles into the same engine core as the standalone plugin path, so
//    Clip without bounds is a no-op (ONNX defaults, -inf/+inf) on both paths; the
//    reference's EP graph defaulted to [0, 1] (src/onnxruntime-hip/hip_graph.h:51-52)
//    while its engine used +-inf (src/vapoursynth/hip_engine.h:47-52).
#pragma once

#include <string>
#include <unordered_map>
#include <vector>

#include "onnx_wire.h"

namespace ah {
namespace ep {

struct Region {
  std::string name;                      // "HipKernel_graph_<k>", k from a process-wide counter
  std::vector<int> nodes;                // positions in graph.nodes, in node order
  std::vector<std::string> activations;  // external non-initializer inputs (exactly one when claimed)
  std::vector<std::string> constants;    // external initializer inputs
  std::vector<std::string> outputs;      // values needed outside the run (exactly one when claimed)
};

// Element type of every value the graph names (graph inputs, initializers, node outputs);
// 0 where it cannot be inferred.
std::unordered_map<std::string, int> InferElemTypes(const onnx::Graph& g);

// IsNodeSupported for node `index` of the graph.
bool IsNodeSupported(const onnx::Graph& g, int index, const std::unordered_map<std::string, int>& types);

// GetCapability: the claimed runs (each with one activation input and one output). Empty
// when the provider has no usable device context (`context_ok` false), as the reference
// refuses every node then.
std::vector<Region> GetCapability(const onnx::Model& m, bool context_ok);

// The standalone model of a claimed run: its nodes in order, the activation as the single
// graph input, the output as the single graph output (types inferred; the shape is taken
// from the graph's declaration when the value is a graph input or output), the constants as
// initializers. What Compile hands to the engine.
onnx::Model RegionModel(const onnx::Model& m, const Region& r);

}  // namespace ep
}  // namespace ah
