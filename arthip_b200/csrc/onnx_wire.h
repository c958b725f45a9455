// Self-contained ONNX ModelProto decoder (protobuf wire format; no libonnx/libprotobuf).
//
// Decodes the subset of onnx.proto the conv-chain engine consumes: graph nodes with
// their attributes, initializers (raw_data and the typed float/int32/int64/double
// fields, data_location) and the graph input/output value infos. The reference parses
// the same fields through the generated protobuf classes (src/vapoursynth/onnx_utils.cpp:29-93,
// src/vapoursynth/hip_engine.cc:51-112).
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace ah {
namespace onnx {

enum DataType : int {
  kUndefined = 0,
  kFloat = 1,
  kUint8 = 2,
  kInt8 = 3,
  kUint16 = 4,
  kInt16 = 5,
  kInt32 = 6,
  kInt64 = 7,
  kString = 8,
  kBool = 9,
  kFloat16 = 10,
  kDouble = 11,
  kUint32 = 12,
  kUint64 = 13,
  kBfloat16 = 16,
};

enum AttrType : int { kAttrFloat = 1, kAttrInt = 2, kAttrString = 3, kAttrTensor = 4, kAttrFloats = 6, kAttrInts = 7 };

struct Tensor {
  std::string name;
  int data_type = 0;
  std::vector<int64_t> dims;
  std::string raw_data;
  bool has_raw = false;
  std::vector<float> float_data;
  std::vector<int32_t> int32_data;
  std::vector<int64_t> int64_data;
  std::vector<double> double_data;
  bool external = false;
};

struct Attribute {
  std::string name;
  int type = 0;
  float f = 0.f;
  int64_t i = 0;
  std::string s;
  std::vector<float> floats;
  std::vector<int64_t> ints;
  bool has_i = false, has_f = false, has_s = false;
};

struct Node {
  std::string op_type;
  std::string domain;
  std::string name;
  std::vector<std::string> inputs;
  std::vector<std::string> outputs;
  std::vector<Attribute> attrs;
  const Attribute* attr(const std::string& n) const {
    for (const auto& a : attrs)
      if (a.name == n) return &a;
    return nullptr;
  }
};

struct ValueInfo {
  std::string name;
  int elem_type = 0;
  std::vector<int64_t> dims;  // -1 for symbolic / unknown
};

struct Graph {
  std::vector<Node> nodes;
  std::vector<Tensor> initializers;
  std::vector<ValueInfo> inputs;
  std::vector<ValueInfo> outputs;
};

struct Model {
  int64_t ir_version = 0;
  int64_t opset = 0;
  Graph graph;
};

// Returns false with a message on malformed input.
bool ParseModel(const uint8_t* data, size_t size, Model* out, std::string* err);
bool LoadModelFile(const std::string& path, Model* out, std::string* err);
// Serializes the same subset (nodes, initializers, graph input/output value infos, the
// default-domain opset); symbolic dims are written as dim_param "?".
std::string EncodeModel(const Model& m);

}  // namespace onnx
}  // namespace ah
