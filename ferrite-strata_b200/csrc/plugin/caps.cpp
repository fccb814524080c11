// The capability table: what the pull `supports` query answers and the
// capability blob advertises.  Encoding restates
// crates/ferrite-strata-plugin-api/src/wire/caps.rs:66-118; lookup semantics
// follow crates/ferrite-strata/src/capabilities.rs:466-490 (dtype mask gate,
// then the table, refusal by default).
#include "plugin.hpp"

namespace sbp {

namespace {

constexpr uint32_t F32 = STRATA_ELEM_F32, BF16 = STRATA_ELEM_BF16;

struct PatternRule {
  const char* id;
  bool fused;  // Fused for vendor patterns, Fallback for single reference ops
  // Output dtypes accepted (the partitioner asks with the first output's dtype,
  // crates/ferrite-strata/src/partition.rs:532-547).
  bool f32, bf16, i32_ids, u8_w4, i8_w8;
};

const PatternRule kRules[] = {
    // The twelve reference ops (capabilities.rs:562-627), each run as its own kernel.
    {"ref::add", false, true, true, false, false, false},
    {"ref::mul", false, true, true, false, false, false},
    {"ref::matmul", false, true, false, false, false, false},
    {"ref::log", false, true, true, false, false, false},
    {"ref::exp", false, true, true, false, false, false},
    {"ref::softmax", false, true, true, false, false, false},
    {"ref::layer_norm", false, true, true, false, false, false},
    {"ref::gelu", false, true, true, false, false, false},
    {"ref::linear", false, true, true, false, false, false},
    {"ref::reshape", false, true, true, false, false, false},
    {"ref::transpose", false, true, true, false, false, false},
    {"ref::expand", false, true, true, false, false, false},
    // The decoder-block patterns this backend fuses.
    {"fused::linear_w4g32", true, false, true, false, false, false},
    {"fused::linear_w8pc", true, false, true, false, false, false},
    {"fused::linear_mxfp8", true, false, true, false, false, false},
    {"fused::linear_mxfp4", true, false, true, false, false, false},
    {"fused::rms_norm", true, true, true, false, false, false},
    {"fused::rope", true, true, true, false, false, false},
    {"fused::swiglu", true, true, true, false, false, false},
    {"fused::attention", true, true, true, false, false, false},
    {"fused::embed", true, true, true, false, false, false},
    {"fused::argmax", true, false, false, true, false, false},
    {"fused::vocab_argmax", true, false, false, true, false, false},
    {"fused::all_reduce", true, true, true, false, false, false},
    {"fused::last_token", true, true, true, false, false, false},
    {"fused::quantize_w4g32", true, false, false, false, true, false},
    {"fused::quantize_w8pc", true, false, false, false, false, true},
    {"fused::dequantize_w4g32", true, true, false, false, false, false},
    {"fused::dequantize_w8pc", true, true, false, false, false, false},
};

bool dtype_ok(const PatternRule& r, const DType& d) {
  if (d.elem == F32 && d.qkind == 0) return r.f32;
  if (d.elem == BF16 && d.qkind == 0) return r.bf16;
  if (d.elem == STRATA_ELEM_I32 && d.qkind == STRATA_QUANT_BLOCK) return r.i32_ids;
  if (d.elem == STRATA_ELEM_U8 && d.qkind == STRATA_QUANT_BLOCK && d.block == 32 && d.sym) return r.u8_w4;
  if (d.elem == STRATA_ELEM_I8 && d.qkind == STRATA_QUANT_BLOCK && d.sym) return r.i8_w8;
  return false;
}

bool shape_ok(uint32_t kind, uint8_t rank) {
  if (kind <= STRATA_SHAPE_BATCH4) return true;
  return kind == STRATA_SHAPE_HIGHER_RANK && rank >= 5 && rank <= kMaxRank;
}

// DTypeMask bits are positions in ElementType::all() (dtype.rs:156-173).
uint32_t mask_bit(uint32_t abi_elem) {
  switch (abi_elem) {
    case STRATA_ELEM_F32: return 1u << 3;
    case STRATA_ELEM_BF16: return 1u << 5;
    case STRATA_ELEM_I8: return 1u << 8;
    case STRATA_ELEM_I32: return 1u << 10;
    case STRATA_ELEM_U8: return 1u << 12;
    case STRATA_ELEM_F8E4M3: return 1u << 1;
    case STRATA_ELEM_F8E8M0: return 1u << 6;
    case STRATA_ELEM_F4E2M1: return 1u << 7;
  }
  return 0;
}

}  // namespace

uint32_t supports_query(const std::string& pattern, const DType& dt, uint32_t shape_kind,
                        uint8_t shape_rank) {
  if (!shape_ok(shape_kind, shape_rank)) return STRATA_SUPPORT_REFUSE;
  for (const auto& r : kRules) {
    if (pattern != r.id) continue;
    if (!dtype_ok(r, dt)) return STRATA_SUPPORT_REFUSE;
    return r.fused ? STRATA_SUPPORT_FUSED : STRATA_SUPPORT_FALLBACK;
  }
  return STRATA_SUPPORT_REFUSE;
}

std::vector<uint8_t> build_caps(const Ctx& ctx) {
  Writer w;
  w.u32(kCapsSchema);
  w.str("b200");
  struct Entry {
    std::string id;
    DType dt;
    uint32_t kind;
    uint8_t rank;
    uint32_t level;
    const char* reason;
  };
  std::vector<Entry> entries;
  std::vector<std::pair<uint32_t, uint8_t>> classes;
  for (uint32_t k = STRATA_SHAPE_SCALAR; k <= STRATA_SHAPE_BATCH4; ++k) classes.push_back({k, 0});
  for (uint8_t r = 5; r <= kMaxRank; ++r) classes.push_back({STRATA_SHAPE_HIGHER_RANK, r});
  for (const auto& r : kRules) {
    std::vector<std::pair<DType, const char*>> dts;
    DType d;
    if (r.f32) d = DType{F32, 0, 0, 0}, dts.push_back({d, nullptr});
    if (r.bf16) d = DType{BF16, 0, 0, 0}, dts.push_back({d, nullptr});
    if (r.i32_ids)
      d = DType{STRATA_ELEM_I32, STRATA_QUANT_BLOCK, 1, 1},
      dts.push_back({d, "integer ids; any block_size is accepted"});
    if (r.u8_w4)
      d = DType{STRATA_ELEM_U8, STRATA_QUANT_BLOCK, 32, 1},
      dts.push_back({d, "int4 codes, two per byte, low nibble = even k"});
    if (r.i8_w8)
      d = DType{STRATA_ELEM_I8, STRATA_QUANT_BLOCK, 4096, 1},
      dts.push_back({d, "int8 per output channel; block_size = K, any K"});
    for (const auto& dd : dts)
      for (const auto& c : classes)
        entries.push_back({r.id, dd.first, c.first, c.second,
                           r.fused ? STRATA_SUPPORT_FUSED : STRATA_SUPPORT_FALLBACK, dd.second});
  }
  w.u32(uint32_t(entries.size()));
  for (const auto& e : entries) {
    w.str(e.id);
    w.u32(e.dt.elem);
    w.u32(e.dt.qkind);
    w.u32(e.dt.block);
    w.u8(e.dt.sym);
    w.u32(e.kind);
    w.u8(e.rank);
    w.u32(e.level);
    if (e.reason) {
      w.u8(1);
      w.str(e.reason);
    } else {
      w.u8(0);
    }
  }
  // One compute unit: the device this context drives.
  w.u32(1);
  w.u32(uint32_t(ctx.device));
  w.str(ctx.device_name);
  w.str("gpu");
  if (ctx.memory_bytes) {
    w.u8(1);
    w.u64(ctx.memory_bytes);
  } else {
    w.u8(0);
  }
  w.u64(ctx.memory_bytes ? ctx.memory_bytes : ~uint64_t(0));  // max_allocation_bytes
  w.u64(~uint64_t(0));                                         // max_graph_bytes
  w.u32(uint32_t(kMaxRank));                                   // max_rank
  w.u64(~uint64_t(0));                                         // max_dim
  w.u64(~uint64_t(0));                                         // max_nodes
  // Tensors of these element types can reach a compiled graph (the MX
  // formats as linear weights and scales).
  w.u32(mask_bit(F32) | mask_bit(BF16) | mask_bit(STRATA_ELEM_I8) | mask_bit(STRATA_ELEM_I32) |
        mask_bit(STRATA_ELEM_U8) | mask_bit(STRATA_ELEM_F8E4M3) | mask_bit(STRATA_ELEM_F8E8M0) |
        mask_bit(STRATA_ELEM_F4E2M1));
  w.u8(1);  // accepts_unpartitioned
  return std::move(w.data());
}

}  // namespace sbp
