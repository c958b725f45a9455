// Protobuf wire-format decoder for the ONNX subset in onnx_wire.h.
#include "onnx_wire.h"

#include <cstdio>
#include <cstring>

namespace ah {
namespace onnx {

namespace {

class Reader {
 public:
  Reader(const uint8_t* p, size_t n) : p_(p), end_(p + n) {}
  bool done() const { return p_ >= end_; }

  bool varint(uint64_t* v) {
    uint64_t r = 0;
    for (int shift = 0; shift < 64; shift += 7) {
      if (p_ >= end_) return false;
      const uint8_t b = *p_++;
      r |= static_cast<uint64_t>(b & 0x7F) << shift;
      if (!(b & 0x80)) {
        *v = r;
        return true;
      }
    }
    return false;
  }

  // Reads one field header and its payload. For length-delimited fields `sub` points at
  // the payload; for fixed/varint fields `val` holds the value (fixed32/64 as raw bits).
  bool field(uint32_t* fnum, uint32_t* wtype, uint64_t* val, const uint8_t** sub, size_t* sublen) {
    uint64_t key;
    if (!varint(&key)) return false;
    *fnum = static_cast<uint32_t>(key >> 3);
    *wtype = static_cast<uint32_t>(key & 7);
    switch (*wtype) {
      case 0:
        return varint(val);
      case 1:
        if (end_ - p_ < 8) return false;
        std::memcpy(val, p_, 8);
        p_ += 8;
        return true;
      case 5: {
        if (end_ - p_ < 4) return false;
        uint32_t v32;
        std::memcpy(&v32, p_, 4);
        *val = v32;
        p_ += 4;
        return true;
      }
      case 2: {
        uint64_t len;
        if (!varint(&len)) return false;
        if (static_cast<uint64_t>(end_ - p_) < len) return false;
        *sub = p_;
        *sublen = static_cast<size_t>(len);
        p_ += len;
        return true;
      }
      default:
        return false;  // groups (3/4) are not used by ONNX
    }
  }

 private:
  const uint8_t* p_;
  const uint8_t* end_;
};

std::string Str(const uint8_t* p, size_t n) { return std::string(reinterpret_cast<const char*>(p), n); }

// Appends repeated varint values from either a packed payload or a single varint.
template <typename T>
bool Varints(uint32_t wt, uint64_t val, const uint8_t* sub, size_t n, std::vector<T>* out) {
  if (wt == 0) {
    out->push_back(static_cast<T>(static_cast<int64_t>(val)));
    return true;
  }
  if (wt != 2) return false;
  Reader r(sub, n);
  while (!r.done()) {
    uint64_t v;
    if (!r.varint(&v)) return false;
    out->push_back(static_cast<T>(static_cast<int64_t>(v)));
  }
  return true;
}

bool Floats(uint32_t wt, uint64_t val, const uint8_t* sub, size_t n, std::vector<float>* out) {
  if (wt == 5) {
    uint32_t b = static_cast<uint32_t>(val);
    float f;
    std::memcpy(&f, &b, 4);
    out->push_back(f);
    return true;
  }
  if (wt != 2 || n % 4) return false;
  const size_t k = n / 4;
  const size_t base = out->size();
  out->resize(base + k);
  std::memcpy(out->data() + base, sub, n);
  return true;
}

bool Doubles(uint32_t wt, uint64_t val, const uint8_t* sub, size_t n, std::vector<double>* out) {
  if (wt == 1) {
    double d;
    std::memcpy(&d, &val, 8);
    out->push_back(d);
    return true;
  }
  if (wt != 2 || n % 8) return false;
  const size_t base = out->size();
  out->resize(base + n / 8);
  std::memcpy(out->data() + base, sub, n);
  return true;
}

bool ParseTensor(const uint8_t* p, size_t n, Tensor* t) {
  Reader r(p, n);
  while (!r.done()) {
    uint32_t f, wt;
    uint64_t v = 0;
    const uint8_t* s = nullptr;
    size_t sl = 0;
    if (!r.field(&f, &wt, &v, &s, &sl)) return false;
    switch (f) {
      case 1:
        if (!Varints(wt, v, s, sl, &t->dims)) return false;
        break;
      case 2:
        t->data_type = static_cast<int>(v);
        break;
      case 4:
        if (!Floats(wt, v, s, sl, &t->float_data)) return false;
        break;
      case 5:
        if (!Varints(wt, v, s, sl, &t->int32_data)) return false;
        break;
      case 7:
        if (!Varints(wt, v, s, sl, &t->int64_data)) return false;
        break;
      case 8:
        t->name = Str(s, sl);
        break;
      case 9:
        t->raw_data = Str(s, sl);
        t->has_raw = true;
        break;
      case 10:
        if (!Doubles(wt, v, s, sl, &t->double_data)) return false;
        break;
      case 13:
        t->external = true;  // external_data entries present
        break;
      case 14:
        if (v == 1) t->external = true;
        break;
      default:
        break;
    }
  }
  return true;
}

bool ParseAttr(const uint8_t* p, size_t n, Attribute* a) {
  Reader r(p, n);
  while (!r.done()) {
    uint32_t f, wt;
    uint64_t v = 0;
    const uint8_t* s = nullptr;
    size_t sl = 0;
    if (!r.field(&f, &wt, &v, &s, &sl)) return false;
    switch (f) {
      case 1:
        a->name = Str(s, sl);
        break;
      case 20:
        a->type = static_cast<int>(v);
        break;
      case 2: {
        uint32_t b = static_cast<uint32_t>(v);
        std::memcpy(&a->f, &b, 4);
        a->has_f = true;
        break;
      }
      case 3:
        a->i = static_cast<int64_t>(v);
        a->has_i = true;
        break;
      case 4:
        a->s = Str(s, sl);
        a->has_s = true;
        break;
      case 7:
        if (!Floats(wt, v, s, sl, &a->floats)) return false;
        break;
      case 8:
        if (!Varints(wt, v, s, sl, &a->ints)) return false;
        break;
      default:
        break;
    }
  }
  if (a->type == 0) {
    if (!a->ints.empty()) a->type = kAttrInts;
    else if (!a->floats.empty()) a->type = kAttrFloats;
    else if (a->has_s) a->type = kAttrString;
    else if (a->has_i) a->type = kAttrInt;
    else if (a->has_f) a->type = kAttrFloat;
  }
  return true;
}

bool ParseNode(const uint8_t* p, size_t n, Node* nd) {
  Reader r(p, n);
  while (!r.done()) {
    uint32_t f, wt;
    uint64_t v = 0;
    const uint8_t* s = nullptr;
    size_t sl = 0;
    if (!r.field(&f, &wt, &v, &s, &sl)) return false;
    switch (f) {
      case 1:
        nd->inputs.push_back(Str(s, sl));
        break;
      case 2:
        nd->outputs.push_back(Str(s, sl));
        break;
      case 3:
        nd->name = Str(s, sl);
        break;
      case 4:
        nd->op_type = Str(s, sl);
        break;
      case 5: {
        Attribute a;
        if (!ParseAttr(s, sl, &a)) return false;
        nd->attrs.push_back(std::move(a));
        break;
      }
      case 7:
        nd->domain = Str(s, sl);
        break;
      default:
        break;
    }
  }
  return true;
}

bool ParseValueInfo(const uint8_t* p, size_t n, ValueInfo* vi) {
  Reader r(p, n);
  while (!r.done()) {
    uint32_t f, wt;
    uint64_t v = 0;
    const uint8_t* s = nullptr;
    size_t sl = 0;
    if (!r.field(&f, &wt, &v, &s, &sl)) return false;
    if (f == 1) {
      vi->name = Str(s, sl);
    } else if (f == 2 && wt == 2) {  // TypeProto
      Reader tr(s, sl);
      while (!tr.done()) {
        uint32_t f2, w2;
        uint64_t v2 = 0;
        const uint8_t* s2 = nullptr;
        size_t l2 = 0;
        if (!tr.field(&f2, &w2, &v2, &s2, &l2)) return false;
        if (f2 != 1 || w2 != 2) continue;  // tensor_type
        Reader ttr(s2, l2);
        while (!ttr.done()) {
          uint32_t f3, w3;
          uint64_t v3 = 0;
          const uint8_t* s3 = nullptr;
          size_t l3 = 0;
          if (!ttr.field(&f3, &w3, &v3, &s3, &l3)) return false;
          if (f3 == 1) {
            vi->elem_type = static_cast<int>(v3);
          } else if (f3 == 2 && w3 == 2) {  // TensorShapeProto
            Reader sr(s3, l3);
            while (!sr.done()) {
              uint32_t f4, w4;
              uint64_t v4 = 0;
              const uint8_t* s4 = nullptr;
              size_t l4 = 0;
              if (!sr.field(&f4, &w4, &v4, &s4, &l4)) return false;
              if (f4 != 1 || w4 != 2) continue;
              int64_t d = -1;
              Reader dr(s4, l4);
              while (!dr.done()) {
                uint32_t f5, w5;
                uint64_t v5 = 0;
                const uint8_t* s5 = nullptr;
                size_t l5 = 0;
                if (!dr.field(&f5, &w5, &v5, &s5, &l5)) return false;
                if (f5 == 1 && w5 == 0) d = static_cast<int64_t>(v5);
              }
              vi->dims.push_back(d);
            }
          }
        }
      }
    }
  }
  return true;
}

bool ParseGraph(const uint8_t* p, size_t n, Graph* g) {
  Reader r(p, n);
  while (!r.done()) {
    uint32_t f, wt;
    uint64_t v = 0;
    const uint8_t* s = nullptr;
    size_t sl = 0;
    if (!r.field(&f, &wt, &v, &s, &sl)) return false;
    if (wt != 2) continue;
    if (f == 1) {
      Node nd;
      if (!ParseNode(s, sl, &nd)) return false;
      g->nodes.push_back(std::move(nd));
    } else if (f == 5) {
      Tensor t;
      if (!ParseTensor(s, sl, &t)) return false;
      g->initializers.push_back(std::move(t));
    } else if (f == 11 || f == 12) {
      ValueInfo vi;
      if (!ParseValueInfo(s, sl, &vi)) return false;
      (f == 11 ? g->inputs : g->outputs).push_back(std::move(vi));
    }
  }
  return true;
}

}  // namespace

bool ParseModel(const uint8_t* data, size_t size, Model* out, std::string* err) {
  Reader r(data, size);
  bool have_graph = false;
  while (!r.done()) {
    uint32_t f, wt;
    uint64_t v = 0;
    const uint8_t* s = nullptr;
    size_t sl = 0;
    if (!r.field(&f, &wt, &v, &s, &sl)) {
      if (err) *err = "failed to parse model (malformed protobuf)";
      return false;
    }
    if (f == 1 && wt == 0) {
      out->ir_version = static_cast<int64_t>(v);
    } else if (f == 7 && wt == 2) {
      if (!ParseGraph(s, sl, &out->graph)) {
        if (err) *err = "failed to parse model graph (malformed protobuf)";
        return false;
      }
      have_graph = true;
    } else if (f == 8 && wt == 2) {
      Reader orr(s, sl);
      std::string dom;
      int64_t ver = 0;
      while (!orr.done()) {
        uint32_t f2, w2;
        uint64_t v2 = 0;
        const uint8_t* s2 = nullptr;
        size_t l2 = 0;
        if (!orr.field(&f2, &w2, &v2, &s2, &l2)) break;
        if (f2 == 1) dom = Str(s2, l2);
        else if (f2 == 2) ver = static_cast<int64_t>(v2);
      }
      if (dom.empty() || dom == "ai.onnx") out->opset = ver;
    }
  }
  if (!have_graph) {
    if (err) *err = "failed to parse model file (no graph)";
    return false;
  }
  // Older exporters list initializers among the graph inputs; those are not activations.
  std::vector<ValueInfo> acts;
  for (const auto& vi : out->graph.inputs) {
    bool is_init = false;
    for (const auto& t : out->graph.initializers)
      if (t.name == vi.name) is_init = true;
    if (!is_init) acts.push_back(vi);
  }
  if (!acts.empty()) out->graph.inputs.swap(acts);
  return true;
}

bool LoadModelFile(const std::string& path, Model* out, std::string* err) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) {
    if (err) *err = "failed to parse model file (cannot open '" + path + "')";
    return false;
  }
  std::vector<uint8_t> buf;
  uint8_t tmp[1 << 16];
  size_t n;
  while ((n = std::fread(tmp, 1, sizeof(tmp), f)) > 0) buf.insert(buf.end(), tmp, tmp + n);
  std::fclose(f);
  return ParseModel(buf.data(), buf.size(), out, err);
}

// ---------------------------------------------------------------------------
// Encoder (the same subset): used to hand a converted model back to a caller.
// ---------------------------------------------------------------------------
namespace {

void PutVarint(std::string* o, uint64_t v) {
  while (v >= 0x80) {
    o->push_back(static_cast<char>((v & 0x7F) | 0x80));
    v >>= 7;
  }
  o->push_back(static_cast<char>(v));
}
void PutKey(std::string* o, uint32_t f, uint32_t wt) { PutVarint(o, (static_cast<uint64_t>(f) << 3) | wt); }
void PutInt(std::string* o, uint32_t f, int64_t v) {
  PutKey(o, f, 0);
  PutVarint(o, static_cast<uint64_t>(v));
}
void PutBytes(std::string* o, uint32_t f, const std::string& b) {
  PutKey(o, f, 2);
  PutVarint(o, b.size());
  o->append(b);
}
template <typename T>
void PutPackedVarints(std::string* o, uint32_t f, const std::vector<T>& v) {
  if (v.empty()) return;
  std::string b;
  for (T x : v) PutVarint(&b, static_cast<uint64_t>(static_cast<int64_t>(x)));
  PutBytes(o, f, b);
}
template <typename T>
void PutPackedFixed(std::string* o, uint32_t f, const std::vector<T>& v) {
  if (v.empty()) return;
  PutBytes(o, f, std::string(reinterpret_cast<const char*>(v.data()), v.size() * sizeof(T)));
}

std::string EncTensor(const Tensor& t) {
  std::string o;
  PutPackedVarints(&o, 1, t.dims);
  PutInt(&o, 2, t.data_type);
  PutPackedFixed(&o, 4, t.float_data);
  PutPackedVarints(&o, 5, t.int32_data);
  PutPackedVarints(&o, 7, t.int64_data);
  PutBytes(&o, 8, t.name);
  if (t.has_raw) PutBytes(&o, 9, t.raw_data);
  PutPackedFixed(&o, 10, t.double_data);
  return o;
}

std::string EncAttr(const Attribute& a) {
  std::string o;
  PutBytes(&o, 1, a.name);
  switch (a.type) {
    case kAttrFloat: {
      PutKey(&o, 2, 5);
      uint32_t b;
      std::memcpy(&b, &a.f, 4);
      for (int k = 0; k < 4; ++k) o.push_back(static_cast<char>((b >> (8 * k)) & 0xFF));
      break;
    }
    case kAttrInt: PutInt(&o, 3, a.i); break;
    case kAttrString: PutBytes(&o, 4, a.s); break;
    case kAttrFloats: PutPackedFixed(&o, 7, a.floats); break;
    case kAttrInts: PutPackedVarints(&o, 8, a.ints); break;
    default: break;
  }
  PutInt(&o, 20, a.type);
  return o;
}

std::string EncNode(const Node& n) {
  std::string o;
  for (const auto& i : n.inputs) PutBytes(&o, 1, i);
  for (const auto& i : n.outputs) PutBytes(&o, 2, i);
  if (!n.name.empty()) PutBytes(&o, 3, n.name);
  PutBytes(&o, 4, n.op_type);
  for (const auto& a : n.attrs) PutBytes(&o, 5, EncAttr(a));
  if (!n.domain.empty()) PutBytes(&o, 7, n.domain);
  return o;
}

std::string EncValueInfo(const ValueInfo& v) {
  std::string shape;
  for (int64_t d : v.dims) {
    std::string dim;
    if (d >= 0) PutInt(&dim, 1, d);
    else PutBytes(&dim, 2, "?");
    PutBytes(&shape, 1, dim);
  }
  std::string tt;
  PutInt(&tt, 1, v.elem_type);
  PutBytes(&tt, 2, shape);
  std::string type;
  PutBytes(&type, 1, tt);
  std::string o;
  PutBytes(&o, 1, v.name);
  PutBytes(&o, 2, type);
  return o;
}

}  // namespace

std::string EncodeModel(const Model& m) {
  std::string g;
  for (const auto& n : m.graph.nodes) PutBytes(&g, 1, EncNode(n));
  PutBytes(&g, 2, "arthip_b200");
  for (const auto& t : m.graph.initializers) PutBytes(&g, 5, EncTensor(t));
  for (const auto& v : m.graph.inputs) PutBytes(&g, 11, EncValueInfo(v));
  for (const auto& v : m.graph.outputs) PutBytes(&g, 12, EncValueInfo(v));
  std::string o;
  PutInt(&o, 1, m.ir_version ? m.ir_version : 8);
  PutBytes(&o, 7, g);
  std::string opset;
  PutBytes(&opset, 1, "");
  PutInt(&opset, 2, m.opset ? m.opset : 13);
  PutBytes(&o, 8, opset);
  return o;
}

}  // namespace onnx
}  // namespace ah
