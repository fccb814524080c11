// Wire format: the versioned little-endian blobs that carry a subgraph into
// the plugin and the capability table out of it.
//
// Framing restates crates/ferrite-strata-plugin-api/src/wire/mod.rs:21-39
// (header, section count, section table, payloads); the graph section
// restates wire/graph.rs:5-29, 101-370; the capability section restates
// wire/caps.rs:1-118.  Every length is bounds-checked before it is trusted
// (wire/mod.rs:47-57, Reader::count at :427).
#pragma once

#include <cstdint>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

namespace sbp {

struct WireError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

constexpr uint64_t kMagic = 0x3147415441525453ull;  // "STRATAG1" little-endian
constexpr uint32_t kFormatMajor = 0, kFormatMinor = 1;
constexpr uint32_t kGraphSchema = 1, kCapsSchema = 1;
constexpr uint32_t kSectionGraph = 1, kSectionCaps = 2;
// Ahead-of-time executables: a section of this plugin's own (outside the
// reference's section kinds) that records the build and the lowered plan.
constexpr uint32_t kSectionB200Exe = 0x45583242;  // "B2XE"
constexpr int kMaxRank = 8;

class Reader {
 public:
  Reader(const uint8_t* p, size_t n) : p_(p), n_(n) {}
  size_t remaining() const { return n_ - at_; }
  const uint8_t* take(size_t n);
  uint8_t u8() { return *take(1); }
  uint32_t u32();
  uint64_t u64();
  std::string str();
  // A u32 count checked against the bytes left at min_item bytes per item.
  size_t count(size_t min_item);

 private:
  const uint8_t* p_;
  size_t n_;
  size_t at_ = 0;
};

class Writer {
 public:
  void u8(uint8_t v) { b_.push_back(v); }
  void u32(uint32_t v);
  void u64(uint64_t v);
  void str(const std::string& s);
  void bytes(const uint8_t* p, size_t n) { b_.insert(b_.end(), p, p + n); }
  std::vector<uint8_t>& data() { return b_; }

 private:
  std::vector<uint8_t> b_;
};

struct DType {
  uint32_t elem = 4;  // STRATA_ELEM_*
  uint32_t qkind = 0;
  uint32_t block = 0;
  uint8_t sym = 0;
  bool operator==(const DType& o) const {
    return elem == o.elem && qkind == o.qkind && block == o.block && sym == o.sym;
  }
  size_t elem_bytes() const;
  // Bytes of n elements as stored here: f4e2m1 codes are packed two per byte
  // (the reference's ElementType::size_in_bytes reports 2 per element,
  // dtype.rs; its larger buffers are accepted).
  uint64_t byte_len(uint64_t n) const { return elem == 13 ? (n + 1) / 2 : n * elem_bytes(); }
  bool is_int() const;
};

struct Value {
  DType dt;
  std::vector<int64_t> dims;
  int64_t producer = -1;  // node index, -1 for a graph input
  uint32_t slot = 0;
  std::string name;
  int64_t elements() const {
    int64_t n = 1;
    for (auto d : dims) n *= d;
    return n;
  }
  uint64_t bytes() const { return dt.byte_len(uint64_t(elements())); }
};

struct Attr {
  uint8_t tag = 0;  // 0 int, 1 float, 2 bool, 3 str, 4 ints (wire/graph.rs:82-88)
  int64_t i = 0;
  float f = 0.0f;
  bool b = false;
  std::string s;
  std::vector<int64_t> ints;
};

struct Node {
  uint32_t op = 0;  // STRATA_OP_*
  // Typed op payloads (wire/graph.rs:177-222).
  int64_t axis = 0;
  uint32_t gamma = 0, beta = 0;
  float eps = 0.0f;
  uint32_t weight = 0;
  bool has_bias = false;
  uint32_t bias = 0;
  std::vector<int64_t> shape;  // Reshape / Expand target
  std::vector<int64_t> perm;   // Transpose
  int64_t s_start = 0, s_end = 0, s_stride = 1;
  std::string pattern;  // Custom
  std::vector<uint32_t> inputs, outputs;
  std::map<std::string, Attr> attrs;
  std::string name;

  int64_t attr_int(const char* k, int64_t dflt) const;
  double attr_float(const char* k, double dflt) const;
  bool has_attr(const char* k) const { return attrs.count(k) != 0; }
};

struct Graph {
  std::string name;
  std::vector<Value> values;
  std::vector<Node> nodes;
  std::vector<uint32_t> outputs;
};

// Slice the first section of `kind` out of a framed payload (the bytes after
// the 24-byte header).  Returns false if there is none.
bool find_section(const uint8_t* payload, size_t len, uint32_t kind, const uint8_t** out,
                  size_t* out_len);

// Decode and validate a graph section (wire/graph.rs:233-311 plus the
// Graph::from_parts checks, graph.rs:525-605).
Graph decode_graph(const uint8_t* p, size_t n);
std::vector<uint8_t> encode_graph(const Graph& g);

// A framed payload (count + table + sections) for one section.
std::vector<uint8_t> frame_payload(uint32_t kind, const std::vector<uint8_t>& section);
// The same for several sections, in order.
std::vector<uint8_t> frame_sections(const std::vector<std::pair<uint32_t, std::vector<uint8_t>>>& sections);

}  // namespace sbp
