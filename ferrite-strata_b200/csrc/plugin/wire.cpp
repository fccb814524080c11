// Wire codec; see wire.hpp for the layout citations.
#include "wire.hpp"

#include <cstring>
#include <set>

namespace sbp {

const uint8_t* Reader::take(size_t n) {
  if (n > remaining()) throw WireError("truncated: needed " + std::to_string(n) + " bytes, " +
                                      std::to_string(remaining()) + " available");
  const uint8_t* r = p_ + at_;
  at_ += n;
  return r;
}

uint32_t Reader::u32() {
  const uint8_t* b = take(4);
  return uint32_t(b[0]) | uint32_t(b[1]) << 8 | uint32_t(b[2]) << 16 | uint32_t(b[3]) << 24;
}

uint64_t Reader::u64() {
  const uint64_t lo = u32();
  const uint64_t hi = u32();
  return lo | hi << 32;
}

static bool valid_utf8(const uint8_t* s, size_t n) {
  size_t i = 0;
  while (i < n) {
    const uint8_t c = s[i];
    size_t len = c < 0x80 ? 1 : (c >> 5) == 6 ? 2 : (c >> 4) == 14 ? 3 : (c >> 3) == 30 ? 4 : 0;
    if (len == 0 || i + len > n) return false;
    for (size_t j = 1; j < len; ++j)
      if ((s[i + j] & 0xc0) != 0x80) return false;
    i += len;
  }
  return true;
}

std::string Reader::str() {
  const uint32_t len = u32();
  if (len > remaining())
    throw WireError("length overflow: a string declares " + std::to_string(len) + " bytes, " +
                    std::to_string(remaining()) + " available");
  const uint8_t* b = take(len);
  if (!valid_utf8(b, len)) throw WireError("a string field is not valid UTF-8");
  return std::string(reinterpret_cast<const char*>(b), len);
}

size_t Reader::count(size_t min_item) {
  const uint64_t raw = u32();
  if (raw * min_item > remaining())
    throw WireError("length overflow: a count of " + std::to_string(raw) +
                    " cannot fit in the bytes that remain");
  return size_t(raw);
}

void Writer::u32(uint32_t v) {
  for (int i = 0; i < 4; ++i) b_.push_back(uint8_t(v >> (8 * i)));
}
void Writer::u64(uint64_t v) {
  for (int i = 0; i < 8; ++i) b_.push_back(uint8_t(v >> (8 * i)));
}
void Writer::str(const std::string& s) {
  u32(uint32_t(s.size()));
  bytes(reinterpret_cast<const uint8_t*>(s.data()), s.size());
}

size_t DType::elem_bytes() const {
  switch (elem) {
    case 0: case 2: case 6: case 10: case 11: case 12: return 1;  // f8, i8, u8, bool, e8m0
    case 3: case 7: case 13: case 14: return 2;  // f16, i16, f4e2m1 (reference quirk), bf16
    case 4: case 8: return 4;
    case 5: case 9: return 8;
  }
  return 4;
}

bool DType::is_int() const { return elem == 6 || elem == 7 || elem == 8 || elem == 9 || elem == 10 || elem == 11; }

int64_t Node::attr_int(const char* k, int64_t dflt) const {
  auto it = attrs.find(k);
  if (it == attrs.end()) return dflt;
  if (it->second.tag == 0) return it->second.i;
  if (it->second.tag == 1) return int64_t(it->second.f);
  return dflt;
}

double Node::attr_float(const char* k, double dflt) const {
  auto it = attrs.find(k);
  if (it == attrs.end()) return dflt;
  if (it->second.tag == 1) return it->second.f;
  if (it->second.tag == 0) return double(it->second.i);
  return dflt;
}

// wire/graph.rs:446-475: known element and quant tags, and no bare integers.
static DType read_dtype(Reader& r) {
  DType d;
  d.elem = r.u32();
  d.qkind = r.u32();
  d.block = r.u32();
  d.sym = r.u8();
  if (d.elem == 1 || d.elem > 14) throw WireError("unknown element-type tag " + std::to_string(d.elem));
  if (d.qkind > 2) throw WireError("unknown quant-kind tag " + std::to_string(d.qkind));
  if (d.is_int() && d.qkind == 0)
    throw WireError("an integer element type arrived with no scaling convention");
  return d;
}

static std::vector<int64_t> read_dims(Reader& r) {
  const uint32_t rank = r.u32();
  if (rank > uint32_t(kMaxRank))
    throw WireError("rank " + std::to_string(rank) + " exceeds the limit of 8");
  std::vector<int64_t> dims(rank);
  for (auto& d : dims) {
    const uint64_t v = r.u64();
    if (v > (uint64_t(1) << 62)) throw WireError("a dimension is out of range");
    d = int64_t(v);
  }
  return dims;
}

static std::vector<uint32_t> read_ids(Reader& r) {
  const size_t n = r.count(4);
  std::vector<uint32_t> out(n);
  for (auto& v : out) v = r.u32();
  return out;
}

// attrs.rs:151-178: non-empty, <= 64 bytes, [a-z][a-z0-9_]*.
static bool valid_key(const std::string& k) {
  if (k.empty() || k.size() > 64) return false;
  if (!(k[0] >= 'a' && k[0] <= 'z')) return false;
  for (char c : k)
    if (!((c >= 'a' && c <= 'z') || (c >= '0' && c <= '9') || c == '_')) return false;
  return true;
}

static void read_op(Reader& r, Node& n) {
  n.op = r.u32();
  switch (n.op) {
    case 0: case 1: case 2: case 3: case 4: case 5: case 8: break;
    case 6: n.axis = int64_t(r.u64()); break;
    case 7: {
      n.gamma = r.u32();
      n.beta = r.u32();
      const uint32_t bits = r.u32();
      std::memcpy(&n.eps, &bits, 4);
      break;
    }
    case 9:
      n.weight = r.u32();
      n.has_bias = r.u8() != 0;
      if (n.has_bias) n.bias = r.u32();
      break;
    case 10: case 12: n.shape = read_dims(r); break;
    case 11: {
      const size_t len = r.count(8);
      n.perm.resize(len);
      for (auto& v : n.perm) v = int64_t(r.u64());
      break;
    }
    case 13:
      n.axis = int64_t(r.u64());
      n.s_start = int64_t(r.u64());
      n.s_end = int64_t(r.u64());
      n.s_stride = int64_t(r.u64());
      break;
    case 14: n.pattern = r.str(); break;
    default: throw WireError("unknown op tag " + std::to_string(n.op));
  }
}

Graph decode_graph(const uint8_t* p, size_t len) {
  Reader r(p, len);
  Graph g;
  const uint32_t schema = r.u32();
  if (schema != kGraphSchema) throw WireError("unsupported graph schema " + std::to_string(schema));
  g.name = r.str();
  const size_t nv = r.count(13 + 4 + 8 + 4 + 1);
  g.values.resize(nv);
  for (auto& v : g.values) {
    v.dt = read_dtype(r);
    v.dims = read_dims(r);
    const uint64_t prod = r.u64();
    v.producer = prod == ~uint64_t(0) ? -1 : int64_t(prod & ~(uint64_t(1) << 63));
    v.slot = r.u32();
    v.name = r.str();
  }
  const size_t nn = r.count(4 + 8 + 4 + 1);
  g.nodes.resize(nn);
  for (auto& n : g.nodes) {
    read_op(r, n);
    n.inputs = read_ids(r);
    n.outputs = read_ids(r);
    const size_t na = r.count(2);
    for (size_t i = 0; i < na; ++i) {
      const std::string key = r.str();
      if (!valid_key(key)) throw WireError("attribute key `" + key + "` is not snake_case");
      Attr a;
      a.tag = r.u8();
      switch (a.tag) {
        case 0: a.i = int64_t(r.u64()); break;
        case 1: {
          const uint32_t bits = r.u32();
          std::memcpy(&a.f, &bits, 4);
          break;
        }
        case 2: a.b = r.u8() != 0; break;
        case 3: a.s = r.str(); break;
        case 4: {
          const size_t c = r.count(8);
          a.ints.resize(c);
          for (auto& v : a.ints) v = int64_t(r.u64());
          break;
        }
        default: throw WireError("unknown attr tag " + std::to_string(a.tag));
      }
      n.attrs.emplace(key, a);  // a duplicate key keeps the first value
    }
    n.name = r.str();
  }
  g.outputs = read_ids(r);

  // Graph::from_parts (graph.rs:525-605).
  std::set<std::string> names;
  for (const auto& n : g.nodes) {
    if (!names.insert(n.name).second) throw WireError("duplicate name `" + n.name + "`");
    if (n.op == 0 && !n.inputs.empty()) throw WireError("an input node consumes a value");
  }
  for (const auto& v : g.values) {
    if (!names.insert(v.name).second) throw WireError("duplicate name `" + v.name + "`");
    if (v.producer >= int64_t(g.nodes.size()))
      throw WireError("a value names producer " + std::to_string(v.producer) + ", which does not exist");
  }
  std::vector<bool> produced(g.values.size(), false);
  for (size_t i = 0; i < g.values.size(); ++i) produced[i] = g.values[i].producer < 0;
  for (const auto& n : g.nodes) {
    for (auto in : n.inputs) {
      if (in >= g.values.size()) throw WireError("a node reads unknown value " + std::to_string(in));
      if (!produced[in]) throw WireError("value " + std::to_string(in) + " is used before it is defined");
    }
    for (auto out : n.outputs) {
      if (out >= g.values.size()) throw WireError("a node writes unknown value " + std::to_string(out));
      produced[out] = true;
    }
  }
  std::set<uint32_t> seen;
  for (auto out : g.outputs) {
    if (out >= g.values.size()) throw WireError("graph output " + std::to_string(out) + " does not exist");
    if (!seen.insert(out).second) throw WireError("graph output " + std::to_string(out) + " is listed twice");
  }
  return g;
}

std::vector<uint8_t> encode_graph(const Graph& g) {
  Writer w;
  w.u32(kGraphSchema);
  w.str(g.name);
  w.u32(uint32_t(g.values.size()));
  for (const auto& v : g.values) {
    w.u32(v.dt.elem);
    w.u32(v.dt.qkind);
    w.u32(v.dt.block);
    w.u8(v.dt.sym);
    w.u32(uint32_t(v.dims.size()));
    for (auto d : v.dims) w.u64(uint64_t(d));
    w.u64(v.producer < 0 ? ~uint64_t(0) : (uint64_t(v.producer) | (uint64_t(1) << 63)));
    w.u32(v.slot);
    w.str(v.name);
  }
  w.u32(uint32_t(g.nodes.size()));
  for (const auto& n : g.nodes) {
    w.u32(n.op);
    switch (n.op) {
      case 6: w.u64(uint64_t(n.axis)); break;
      case 7: {
        w.u32(n.gamma);
        w.u32(n.beta);
        uint32_t bits;
        std::memcpy(&bits, &n.eps, 4);
        w.u32(bits);
        break;
      }
      case 9:
        w.u32(n.weight);
        w.u8(n.has_bias ? 1 : 0);
        if (n.has_bias) w.u32(n.bias);
        break;
      case 10: case 12:
        w.u32(uint32_t(n.shape.size()));
        for (auto d : n.shape) w.u64(uint64_t(d));
        break;
      case 11:
        w.u32(uint32_t(n.perm.size()));
        for (auto d : n.perm) w.u64(uint64_t(d));
        break;
      case 13:
        w.u64(uint64_t(n.axis));
        w.u64(uint64_t(n.s_start));
        w.u64(uint64_t(n.s_end));
        w.u64(uint64_t(n.s_stride));
        break;
      case 14: w.str(n.pattern); break;
      default: break;
    }
    w.u32(uint32_t(n.inputs.size()));
    for (auto i : n.inputs) w.u32(i);
    w.u32(uint32_t(n.outputs.size()));
    for (auto o : n.outputs) w.u32(o);
    w.u32(uint32_t(n.attrs.size()));
    for (const auto& kv : n.attrs) {
      w.str(kv.first);
      const Attr& a = kv.second;
      w.u8(a.tag);
      switch (a.tag) {
        case 0: w.u64(uint64_t(a.i)); break;
        case 1: {
          uint32_t bits;
          std::memcpy(&bits, &a.f, 4);
          w.u32(bits);
          break;
        }
        case 2: w.u8(a.b ? 1 : 0); break;
        case 3: w.str(a.s); break;
        case 4:
          w.u32(uint32_t(a.ints.size()));
          for (auto v : a.ints) w.u64(uint64_t(v));
          break;
      }
    }
    w.str(n.name);
  }
  w.u32(uint32_t(g.outputs.size()));
  for (auto o : g.outputs) w.u32(o);
  return std::move(w.data());
}

bool find_section(const uint8_t* payload, size_t len, uint32_t kind, const uint8_t** out,
                  size_t* out_len) {
  Reader t(payload, len);
  const uint32_t count = t.u32();
  for (uint32_t i = 0; i < count; ++i) {
    if (t.remaining() < 20) break;
    const uint32_t k = t.u32();
    const uint64_t off = t.u64();
    const uint64_t n = t.u64();
    if (off <= len && n <= len - off && k == kind) {
      *out = payload + off;
      *out_len = size_t(n);
      return true;
    }
  }
  return false;
}

std::vector<uint8_t> frame_payload(uint32_t kind, const std::vector<uint8_t>& section) {
  Writer w;
  w.u32(1);
  w.u32(kind);
  w.u64(4 + 20);  // offsets are relative to the start of the payload
  w.u64(section.size());
  w.bytes(section.data(), section.size());
  return std::move(w.data());
}

std::vector<uint8_t> frame_sections(const std::vector<std::pair<uint32_t, std::vector<uint8_t>>>& sections) {
  Writer w;
  w.u32(uint32_t(sections.size()));
  uint64_t off = 4 + 20 * uint64_t(sections.size());  // relative to the start of the payload
  for (const auto& s : sections) {
    w.u32(s.first);
    w.u64(off);
    w.u64(s.second.size());
    off += s.second.size();
  }
  for (const auto& s : sections) w.bytes(s.second.data(), s.second.size());
  return std::move(w.data());
}

}  // namespace sbp
