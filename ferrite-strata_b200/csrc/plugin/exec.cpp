// Lowering a decoded subgraph to a list of kernel launches, planning the
// device workspace, and enqueueing the launches (optionally as a CUDA graph).
//
// The reference CPU backend compiles one Step per node and runs them in order
// (crates/ferrite-strata-cpu/src/backend.rs:883-1012, 187-304), publishing
// only the declared outputs.  This lowering keeps those semantics and adds
// the fusions a decoder block needs on the GPU:
//   * linears that share their input x run as one launch (q/k/v);
//   * gate and up linears feeding fused::swiglu become one launch whose
//     epilogue applies SwiGLU (the gate/up activations never reach HBM);
//   * a linear whose only consumer is a residual add writes x + W.x directly.
#include <algorithm>
#include <cstdlib>
#include <cmath>
#include <mutex>
#include <cstdio>
#include <cstring>
#include <map>
#include <type_traits>

#include "plugin.hpp"

namespace sbp {

namespace {

bool is_f32(const DType& d) { return d.elem == STRATA_ELEM_F32 && d.qkind == 0; }
bool is_bf16(const DType& d) { return d.elem == STRATA_ELEM_BF16 && d.qkind == 0; }
bool is_float(const DType& d) { return is_f32(d) || is_bf16(d); }
// Integers travel as I32 tagged with a block spec (bare integers are illegal
// on the wire, wire/graph.rs:466-475).
bool is_i32(const DType& d) { return d.elem == STRATA_ELEM_I32 && d.qkind == STRATA_QUANT_BLOCK; }
bool is_w4(const DType& d) {
  return d.elem == STRATA_ELEM_U8 && d.qkind == STRATA_QUANT_BLOCK && d.block == 32 && d.sym;
}
bool is_w8(const DType& d) { return d.elem == STRATA_ELEM_I8 && d.qkind == STRATA_QUANT_BLOCK && d.sym; }

int64_t last_dim(const Value& v) { return v.dims.empty() ? 1 : v.dims.back(); }
int64_t rows_of(const Value& v) {
  const int64_t l = last_dim(v);
  return l == 0 ? 0 : v.elements() / l;
}

struct Lowerer {
  const Graph& g;
  Exe& exe;
  std::string* reason;
  std::vector<std::vector<int>> cons;
  std::vector<bool> absorbed;
  std::vector<bool> is_output;

  Lowerer(const Graph& gr, Exe& e, std::string* r) : g(gr), exe(e), reason(r) {}

  bool decline(const std::string& why) {
    *reason = why;
    return false;
  }

  // RoPE inverse frequencies theta^(-2j/d), j < d/2, in double with the host
  // pow (the oracle's, oracle/strata_oracle.c ora_rope), stored once among the
  // executable's constants: the kernels read them instead of calling pow per
  // element.  Returns their offset there.
  uint64_t rope_table(double theta, int64_t hd) {
    std::vector<uint8_t>& c = exe.consts;
    const uint64_t off = (c.size() + 7) / 8 * 8;
    c.resize(off + size_t(hd / 2) * sizeof(double));
    for (int64_t j = 0; j < hd / 2; ++j) {
      const double v = std::pow(theta, -2.0 * double(j) / double(hd));
      std::memcpy(c.data() + off + size_t(j) * sizeof(double), &v, sizeof(double));
    }
    return off;
  }

  uint32_t in(const Node& n, size_t i) const {
    if (i >= n.inputs.size())
      fail(STRATA_INVALID_ARGUMENT, "node `" + n.name + "` wants operand " + std::to_string(i) +
                                        " but declares " + std::to_string(n.inputs.size()));
    return n.inputs[i];
  }
  const Value& V(uint32_t id) const { return g.values[id]; }

  int cur_node = -1;
  void push(Step s) {
    if (s.node < 0) s.node = cur_node;
    exe.steps.push_back(std::move(s));
  }

  bool same_dims(uint32_t a, uint32_t b) const { return V(a).dims == V(b).dims; }

  // NumPy broadcast of `a` (and optionally `b`) to the output dims.
  bool bcast(const std::vector<int64_t>& out, uint32_t a, uint32_t b, sb::BcastShape& bs) const {
    const int r = int(out.size());
    if (r > 8) return false;
    bs.rank = r;
    bs.total = 1;
    for (int ax = 0; ax < r; ++ax) {
      bs.dims[ax] = out[ax];
      bs.total *= out[ax];
    }
    auto fill = [&](uint32_t id, int64_t* st) {
      const auto& d = V(id).dims;
      const int off = r - int(d.size());
      if (off < 0) return false;
      int64_t stride = 1;
      for (int ax = r - 1; ax >= 0; --ax) {
        const int sa = ax - off;
        if (sa < 0) {
          st[ax] = 0;
          continue;
        }
        if (d[sa] != 1 && d[sa] != out[ax]) return false;
        st[ax] = d[sa] == 1 ? 0 : stride;
        stride *= d[sa];
      }
      return true;
    };
    if (!fill(a, bs.sa)) return false;
    if (b != kNone && !fill(b, bs.sb)) return false;
    return true;
  }

  bool is_linear(const Node& n) const {
    return n.op == STRATA_OP_CUSTOM &&
           (n.pattern == "fused::linear_w4g32" || n.pattern == "fused::linear_w8pc" ||
            n.pattern == "fused::linear_mxfp8" || n.pattern == "fused::linear_mxfp4");
  }

  static sb::WFormat linear_format(const std::string& pattern) {
    if (pattern == "fused::linear_w4g32") return sb::WFormat::W4G32;
    if (pattern == "fused::linear_mxfp8") return sb::WFormat::MXFP8;
    if (pattern == "fused::linear_mxfp4") return sb::WFormat::MXFP4;
    return sb::WFormat::W8PC;
  }

  bool linear_shapes(const Node& n, int64_t& M, int64_t& K, int64_t& N, std::string* why) const {
    const uint32_t x = n.inputs[0], w = n.inputs[1], s = n.inputs[2], y = n.outputs[0];
    const sb::WFormat fmt = linear_format(n.pattern);
    const bool w4 = fmt == sb::WFormat::W4G32;
    const bool mx = fmt == sb::WFormat::MXFP8 || fmt == sb::WFormat::MXFP4;
    if (!is_bf16(V(x).dt) || !is_bf16(V(y).dt)) {
      *why = "quantised linears take and return bf16";
      return false;
    }
    K = last_dim(V(x));
    M = rows_of(V(x));
    N = last_dim(V(y));
    if (rows_of(V(y)) != M) {
      *why = "linear output rows do not match input rows";
      return false;
    }
    if (mx) {
      // MX (dtype.rs DType::microscaled): E4M3 codes [N, K], or E2M1 codes
      // [N, K] (stored two per byte); E8M0 scales [N, K/32].  The decode
      // GEMV copies the scales 4 groups at a time: K % 128 == 0.
      const uint32_t want = fmt == sb::WFormat::MXFP8 ? STRATA_ELEM_F8E4M3 : STRATA_ELEM_F4E2M1;
      if (V(w).dt.elem != want || V(w).dims != std::vector<int64_t>{N, K} || K % 128) {
        *why = "MX weights must be f8e4m3 (mxfp8) or f4e2m1 (mxfp4) codes of shape [N, K] with K % 128 == 0";
        return false;
      }
      if (V(s).dt.elem != STRATA_ELEM_F8E8M0 || V(s).dims != std::vector<int64_t>{N, K / 32}) {
        *why = "MX scales must be f8e8m0 [N, K/32]";
        return false;
      }
      if (N % 16) {
        *why = "MX linears need output features in multiples of 16";
        return false;
      }
    } else if (w4) {
      if (!is_w4(V(w).dt) || V(w).dims != std::vector<int64_t>{N, K / 2} || K % 32) {
        *why = "int4 weights must be U8 Block{32, symmetric} of shape [N, K/2] with K % 32 == 0";
        return false;
      }
      if (!is_bf16(V(s).dt) || V(s).dims != std::vector<int64_t>{N, K / 32}) {
        *why = "int4 scales must be bf16 [N, K/32]";
        return false;
      }
    } else {
      if (!is_w8(V(w).dt) || V(w).dims != std::vector<int64_t>{N, K} || K % 16) {
        *why = "int8 weights must be I8 Block{K, symmetric} of shape [N, K] with K % 16 == 0";
        return false;
      }
      if (!is_f32(V(s).dt) || V(s).dims != std::vector<int64_t>{N}) {
        *why = "int8 scales must be f32 [N]";
        return false;
      }
    }
    if (N % 2) {
      *why = "output features must be even";
      return false;
    }
    return true;
  }

  void add_linear_job(Step& st, const Node& n, uint32_t y, uint32_t r) {
    st.v.push_back(n.inputs[1]);
    st.v.push_back(n.inputs[2]);
    st.v.push_back(y);
    st.v.push_back(r);
    st.reads.push_back(n.inputs[1]);
    st.reads.push_back(n.inputs[2]);
    if (r != kNone) st.reads.push_back(r);
    st.writes.push_back(y);
    st.njobs++;
  }

  Step linear_step(const Node& n, int64_t M, int64_t K) {
    Step st;
    st.kind = SK::Linear;
    st.bf16 = true;
    st.fmt = linear_format(n.pattern);
    st.i[0] = M;
    st.i[1] = K;
    st.v.push_back(n.inputs[0]);
    st.reads.push_back(n.inputs[0]);
    st.label = n.name;
    return st;
  }

  int producer(uint32_t v) const { return int(V(v).producer); }

  bool lower_all() {
    const size_t nv = g.values.size(), nn = g.nodes.size();
    cons.assign(nv, {});
    is_output.assign(nv, false);
    absorbed.assign(nn, false);
    for (auto o : g.outputs) is_output[o] = true;
    for (size_t i = 0; i < nn; ++i) {
      const Node& n = g.nodes[i];
      const bool bad_field =
          (n.op == STRATA_OP_LINEAR && (n.weight >= nv || (n.has_bias && n.bias >= nv))) ||
          (n.op == STRATA_OP_LAYER_NORM && (n.gamma >= nv || n.beta >= nv));
      if (bad_field)
        fail(STRATA_INVALID_ARGUMENT, "node `" + n.name + "` names a weight value that does not exist");
      for (auto v : n.inputs) cons[v].push_back(int(i));
      if (n.op == STRATA_OP_LINEAR) {
        cons[n.weight].push_back(int(i));
        if (n.has_bias) cons[n.bias].push_back(int(i));
      }
      if (n.op == STRATA_OP_LAYER_NORM) {
        cons[n.gamma].push_back(int(i));
        cons[n.beta].push_back(int(i));
      }
      for (auto v : n.outputs)
        if (g.values[v].producer != int64_t(i))
          fail(STRATA_INVALID_ARGUMENT, "value `" + g.values[v].name + "` is written by node `" +
                                            n.name + "` but names another producer");
    }
    if (g.outputs.empty()) return decline("a subgraph with no outputs has nothing to run");

    exe.alias.resize(nv);
    for (size_t v = 0; v < nv; ++v) exe.alias[v] = uint32_t(v);

    for (size_t i = 0; i < nn; ++i) {
      if (absorbed[i]) continue;
      cur_node = int(i);
      if (!lower_node(int(i))) return false;
    }
    fuse_qkv_rope();
    plan_gemm_scratch();
    return true;
  }

  // Linear steps over more than kGemvMaxRows rows run as tcgen05 GEMMs over
  // bf16 weights: scratch for one job's expanded weights [n, k], or for both
  // the gate and the up matrix of a SwiGLU pair (one GEMM with a SwiGLU
  // epilogue).
  void plan_gemm_scratch() {
    for (Step& st : exe.steps) {
      if (st.kind != SK::Linear || st.i[0] <= sb::kGemvMaxRows) continue;
      uint64_t wmax = 0;
      for (int j = 0; j < st.njobs; ++j) {
        const Value& wv = g.values[st.v[1 + 4 * j]];
        const uint64_t n = uint64_t(wv.dims[0]);
        wmax = std::max<uint64_t>(wmax, n * uint64_t(st.i[1]) * 2);
      }
      // One expanded weight matrix; a SwiGLU pair keeps gate and up expanded at once.
      const uint64_t bytes = (wmax + 255) / 256 * 256;
      st.scratch_bytes = st.epi == sb::Epilogue::SwiGLU ? 2 * bytes : bytes;
    }
  }

  // q/k/v linears of one x whose outputs feed only rope(q), rope(k) and one
  // attention node become one launch: the GEMV epilogue rotates q and k and
  // appends k and v to the caches, and the attention step skips its append.
  void fuse_qkv_rope() {
    auto only = [&](uint32_t v, int node) {
      return cons[v].size() == 1 && cons[v][0] == node && !is_output[v];
    };
    auto find_step = [&](SK kind, int node) {
      for (size_t i = 0; i < exe.steps.size(); ++i)
        if (exe.steps[i].kind == kind && exe.steps[i].node == node) return int(i);
      return -1;
    };
    for (size_t si = 0; si < exe.steps.size(); ++si) {
      Step& L = exe.steps[si];
      if (L.kind != SK::Linear || L.njobs != 3 || L.epi != sb::Epilogue::None ||
          L.fmt == sb::WFormat::BF16 || L.i[0] > sb::kGemvMaxRows)
        continue;  // prefill-sized batches keep separate GEMM, rope and append steps
      const uint32_t yq = L.v[3], yk = L.v[7], yv = L.v[11];
      if (cons[yq].size() != 1 || cons[yk].size() != 1 || cons[yv].size() != 1) continue;
      const int rq = cons[yq][0], rk = cons[yk][0], an = cons[yv][0];
      const Node& RQ = g.nodes[rq];
      const Node& RK = g.nodes[rk];
      const Node& A = g.nodes[an];
      auto is_rope = [](const Node& n) { return n.op == STRATA_OP_CUSTOM && n.pattern == "fused::rope"; };
      if (!is_rope(RQ) || !is_rope(RK) || !(A.op == STRATA_OP_CUSTOM && A.pattern == "fused::attention"))
        continue;
      if (RQ.outputs.size() != 1 || RK.outputs.size() != 1 || A.inputs.size() < 6) continue;
      const uint32_t qr = RQ.outputs[0], kr = RK.outputs[0];
      if (!only(yq, rq) || !only(yk, rk) || !only(kr, an) || !only(yv, an) || !only(qr, an)) continue;
      if (A.inputs[0] != qr || A.inputs[1] != kr || A.inputs[2] != yv) continue;
      if (RQ.inputs[1] != A.inputs[5] || RK.inputs[1] != A.inputs[5]) continue;
      const int64_t hd = RQ.attr_int("head_dim", 0);
      if (hd != RK.attr_int("head_dim", 0) || RQ.attr_float("theta", 10000.0) != RK.attr_float("theta", 10000.0))
        continue;
      const int ap = find_step(SK::Attention, an), kp = find_step(SK::KvAppend, an);
      const int sq = find_step(SK::Rope, rq), sk = find_step(SK::Rope, rk);
      if (ap < 0 || kp < 0 || sq < 0 || sk < 0) continue;
      const Step& AT = exe.steps[ap];
      if (!AT.bf16 || AT.i[4] != hd) continue;
      Step f;
      f.kind = SK::QkvRope;
      f.bf16 = true;
      f.fmt = L.fmt;
      f.node = L.node;
      f.label = L.label + "+rope+kv_append";
      f.i[0] = L.i[0];       // M
      f.i[1] = L.i[1];       // K
      f.i[2] = AT.i[2];      // heads
      f.i[3] = AT.i[3];      // kv heads
      f.i[4] = hd;
      f.i[5] = AT.i[5];      // max_len
      f.i[6] = AT.i[1];      // tokens per sequence
      f.d = RQ.attr_float("theta", 10000.0);
      f.const_off = exe.steps[sq].const_off;  // the q RoPE's table (same theta and head_dim)
      const uint32_t kc = A.inputs[3], vc = A.inputs[4], pos = A.inputs[5];
      f.v = {L.v[0], L.v[1], L.v[2], L.v[5], L.v[6], L.v[9], L.v[10], qr, kc, vc, pos};
      f.reads = {L.v[0], L.v[1], L.v[2], L.v[5], L.v[6], L.v[9], L.v[10], pos, kc, vc};
      f.writes = {qr, kc, vc};
      f.i[7] = AT.i[7];  // paged caches: page size, pages per sequence, pages, then the table
      f.i[8] = AT.i[8];
      f.i[9] = AT.i[9];
      if (AT.i[7] > 0) {
        f.v.push_back(AT.v[5]);
        f.reads.push_back(AT.v[5]);
      }
      exe.steps[si] = f;
      std::vector<int> drop = {sq, sk, kp};
      std::sort(drop.rbegin(), drop.rend());
      for (int d : drop) exe.steps.erase(exe.steps.begin() + d);
    }
  }

  bool lower_linear(int ni) {
    const Node& n = g.nodes[ni];
    in(n, 2);
    if (n.outputs.size() != 1) return decline("a quantised linear has exactly one output");
    int64_t M, K, N;
    std::string why;
    if (!linear_shapes(n, M, K, N, &why)) return decline(why);
    const uint32_t x = n.inputs[0], y = n.outputs[0];

    // SwiGLU: silu(gate) * up where gate and up are linears of the same x.
    if (cons[y].size() == 1 && !is_output[y]) {
      const int si = cons[y][0];
      const Node& S = g.nodes[si];
      if (!absorbed[si] && S.op == STRATA_OP_CUSTOM && S.pattern == "fused::swiglu" &&
          S.inputs.size() == 2 && S.outputs.size() == 1 && S.inputs[0] != S.inputs[1] &&
          is_bf16(V(S.outputs[0]).dt)) {
        const uint32_t other = S.inputs[0] == y ? S.inputs[1] : S.inputs[0];
        const int pj = producer(other);
        if (pj >= 0 && pj != ni && !absorbed[pj] && is_linear(g.nodes[pj]) &&
            g.nodes[pj].pattern == n.pattern && g.nodes[pj].inputs.size() >= 3 &&
            g.nodes[pj].inputs[0] == x && cons[other].size() == 1 && !is_output[other]) {
          int64_t M2, K2, N2;
          if (linear_shapes(g.nodes[pj], M2, K2, N2, &why) && N2 == N && K2 == K &&
              V(S.outputs[0]).dims == V(y).dims) {
            const Node& gate = S.inputs[0] == y ? n : g.nodes[pj];
            const Node& up = S.inputs[0] == y ? g.nodes[pj] : n;
            Step st = linear_step(n, M, K);
            st.epi = sb::Epilogue::SwiGLU;
            add_linear_job(st, gate, S.outputs[0], kNone);
            add_linear_job(st, up, kNone, kNone);
            st.writes.pop_back();  // the up job writes nothing
            st.label = S.name;
            push(std::move(st));
            absorbed[ni] = absorbed[pj] = absorbed[si] = true;
            return true;
          }
        }
      }
      // Residual: y + r with r already computed.
      if (!absorbed[si] && S.op == STRATA_OP_ADD && S.inputs.size() == 2 && S.outputs.size() == 1 &&
          S.inputs[0] != S.inputs[1]) {
        const uint32_t r = S.inputs[0] == y ? S.inputs[1] : S.inputs[0];
        const int pr = producer(r);
        if (is_bf16(V(r).dt) && same_dims(r, y) && V(S.outputs[0]).dims == V(y).dims &&
            is_bf16(V(S.outputs[0]).dt) && (pr < 0 || pr < ni)) {
          Step st = linear_step(n, M, K);
          st.epi = sb::Epilogue::Residual;
          add_linear_job(st, n, S.outputs[0], r);
          st.label = n.name + "+" + S.name;
          push(std::move(st));
          absorbed[ni] = absorbed[si] = true;
          return true;
        }
      }
    }

    // Group with later linears of the same x that are not fused otherwise.
    Step st = linear_step(n, M, K);
    add_linear_job(st, n, y, kNone);
    absorbed[ni] = true;
    for (size_t j = ni + 1; j < g.nodes.size() && st.njobs < sb::kMaxJobs; ++j) {
      const Node& o = g.nodes[j];
      if (absorbed[j] || !is_linear(o) || o.pattern != n.pattern || o.inputs.size() < 3 ||
          o.inputs[0] != x || o.outputs.size() != 1)
        continue;
      int64_t M2, K2, N2;
      if (!linear_shapes(o, M2, K2, N2, &why)) continue;
      if (would_fuse(int(j))) continue;
      add_linear_job(st, o, o.outputs[0], kNone);
      absorbed[j] = true;
    }
    push(std::move(st));
    return true;
  }

  // The residual of a tensor-parallel layer: all_reduce(x) -> add(r, .) ->
  // rms_norm(., gamma) becomes one step that writes the sum h and its norm
  // (h keeps its other readers, the next residual add).  bf16 only.
  bool lower_allreduce_add_norm(int ni) {
    const Node& n = g.nodes[ni];
    const uint32_t x = n.inputs[0], a = n.outputs[0];
    if (!is_bf16(V(x).dt) || cons[a].size() != 1 || is_output[a]) return false;
    const int ai = cons[a][0];
    const Node& A = g.nodes[ai];
    if (absorbed[ai] || A.op != STRATA_OP_ADD || A.inputs.size() != 2 || A.outputs.size() != 1 ||
        A.inputs[0] == A.inputs[1])
      return false;
    const uint32_t r = A.inputs[0] == a ? A.inputs[1] : A.inputs[0], h = A.outputs[0];
    const int pr = producer(r);
    if (!is_bf16(V(r).dt) || !is_bf16(V(h).dt) || !same_dims(r, a) || V(h).dims != V(a).dims ||
        !(pr < 0 || pr < ni) || V(h).dims.empty())
      return false;
    for (int ri : cons[h]) {
      const Node& R = g.nodes[size_t(ri)];
      if (absorbed[size_t(ri)] || R.op != STRATA_OP_CUSTOM || R.pattern != "fused::rms_norm" ||
          R.inputs.size() != 2 || R.outputs.size() != 1 || R.inputs[0] != h)
        continue;
      const uint32_t gm = R.inputs[1], y = R.outputs[0];
      const int pg = producer(gm);
      if (!is_bf16(V(gm).dt) || !is_bf16(V(y).dt) || V(y).dims != V(h).dims ||
          V(gm).elements() != last_dim(V(h)) || !(pg < 0 || pg < ni))
        continue;
      Step st;
      st.kind = SK::AllReduceAddNorm;
      st.bf16 = true;
      st.i[0] = rows_of(V(h));
      st.i[1] = last_dim(V(h));
      st.d = R.attr_float("eps", 1e-5);
      if (!bcast(V(h).dims, a, r, st.bs)) return false;
      st.v = {x, r, gm, h, y};
      st.reads = {x, r, gm};
      st.writes = {h, y};
      st.label = n.name + "+" + A.name + "+" + R.name;
      push(std::move(st));
      absorbed[size_t(ni)] = absorbed[size_t(ai)] = absorbed[size_t(ri)] = true;
      return true;
    }
    return false;
  }

  // Whether linear node j will take the SwiGLU or residual path itself.
  bool would_fuse(int j) const {
    const Node& n = g.nodes[j];
    const uint32_t y = n.outputs[0];
    if (cons[y].size() != 1 || is_output[y]) return false;
    const Node& S = g.nodes[cons[y][0]];
    if (S.op == STRATA_OP_CUSTOM && S.pattern == "fused::swiglu") return true;
    if (S.op == STRATA_OP_ADD) return true;
    return false;
  }

  bool float_unary_ok(uint32_t a, uint32_t b) const {
    return is_float(V(a).dt) && V(a).dt == V(b).dt;
  }

  bool lower_node(int ni) {
    const Node& n = g.nodes[ni];
    if (n.op == STRATA_OP_INPUT) return true;
    if (n.outputs.size() != 1 && !(n.op == STRATA_OP_CUSTOM && n.pattern.rfind("fused::quantize_", 0) == 0))
      return decline("every kernel here is single-output; node `" + n.name + "` has " +
                     std::to_string(n.outputs.size()));
    const uint32_t out = n.outputs.empty() ? kNone : n.outputs[0];
    Step st;
    st.label = n.name;
    switch (n.op) {
      case STRATA_OP_ADD:
      case STRATA_OP_MUL: {
        const uint32_t a = in(n, 0), b = in(n, 1);
        if (!is_float(V(out).dt) || !(V(a).dt == V(out).dt) || !(V(b).dt == V(out).dt))
          return decline("add/mul needs matching f32 or bf16 operands");
        st.kind = SK::Binary;
        st.bf16 = is_bf16(V(out).dt);
        st.i[0] = n.op == STRATA_OP_ADD ? 0 : 1;
        if (!bcast(V(out).dims, a, b, st.bs)) return decline("operands do not broadcast to the output");
        st.v = {a, b, out};
        st.reads = {a, b};
        st.writes = {out};
        break;
      }
      case STRATA_OP_MATMUL: {
        const uint32_t a = in(n, 0), b = in(n, 1);
        if (!is_f32(V(a).dt) || !is_f32(V(b).dt) || !is_f32(V(out).dt))
          return decline("matmul runs in f32 only");
        if (V(a).dims.size() != 2 || V(b).dims.size() != 2)
          return decline("matmul is rank-2 only");
        if (V(a).dims[1] != V(b).dims[0])
          fail(STRATA_INVALID_ARGUMENT, "matmul inner dimensions differ: " +
                                            std::to_string(V(a).dims[1]) + " vs " +
                                            std::to_string(V(b).dims[0]));
        st.kind = SK::GemmF32;
        st.i[0] = V(a).dims[0];
        st.i[1] = V(a).dims[1];
        st.i[2] = V(b).dims[1];
        st.i[3] = 0;  // b stored [k, n]
        st.v = {a, b, kNone, out};
        st.reads = {a, b};
        st.writes = {out};
        break;
      }
      case STRATA_OP_LOG:
      case STRATA_OP_EXP:
      case STRATA_OP_GELU: {
        const uint32_t a = in(n, 0);
        if (!float_unary_ok(a, out)) return decline("unary ops need f32 or bf16");
        st.kind = SK::Unary;
        st.bf16 = is_bf16(V(out).dt);
        st.i[0] = n.op == STRATA_OP_GELU ? 0 : (n.op == STRATA_OP_EXP ? 1 : 2);
        st.i[1] = V(out).elements();
        st.v = {a, out};
        st.reads = {a};
        st.writes = {out};
        break;
      }
      case STRATA_OP_SOFTMAX: {
        const uint32_t a = in(n, 0);
        if (!float_unary_ok(a, out)) return decline("softmax needs f32 or bf16");
        const int64_t r = int64_t(V(a).dims.size());
        if (!(n.axis == -1 || n.axis == r - 1)) return decline("softmax over a non-trailing axis");
        st.kind = SK::Softmax;
        st.bf16 = is_bf16(V(out).dt);
        st.i[0] = rows_of(V(a));
        st.i[1] = last_dim(V(a));
        st.v = {a, out};
        st.reads = {a};
        st.writes = {out};
        break;
      }
      case STRATA_OP_LAYER_NORM: {
        const uint32_t a = in(n, 0);
        if (!float_unary_ok(a, out) || !(V(n.gamma).dt == V(a).dt) || !(V(n.beta).dt == V(a).dt))
          return decline("layer norm needs matching f32 or bf16 operands");
        if (V(n.gamma).elements() != last_dim(V(a)) || V(n.beta).elements() != last_dim(V(a)))
          fail(STRATA_INVALID_ARGUMENT, "layer norm gamma/beta do not match the trailing axis");
        st.kind = SK::LayerNorm;
        st.bf16 = is_bf16(V(out).dt);
        st.i[0] = rows_of(V(a));
        st.i[1] = last_dim(V(a));
        st.d = n.eps;
        st.v = {a, n.gamma, n.beta, out};
        st.reads = {a, n.gamma, n.beta};
        st.writes = {out};
        break;
      }
      case STRATA_OP_LINEAR: {
        const uint32_t a = in(n, 0);
        const uint32_t w = n.weight;
        if (w >= g.values.size() || (n.has_bias && n.bias >= g.values.size()))
          fail(STRATA_INVALID_ARGUMENT, "linear names a weight or bias that does not exist");
        const int64_t K = last_dim(V(a)), M = rows_of(V(a));
        if (V(w).dims.size() != 2) return decline("linear weight must be rank 2");
        const int64_t N = V(w).dims[0];
        if (V(w).dims[1] != K)
          fail(STRATA_INVALID_ARGUMENT, "linear inner dimensions differ: " + std::to_string(K) +
                                            " vs " + std::to_string(V(w).dims[1]));
        if (is_f32(V(a).dt) && is_f32(V(w).dt) && is_f32(V(out).dt) &&
            (!n.has_bias || is_f32(V(n.bias).dt))) {
          st.kind = SK::GemmF32;
          st.i[0] = M;
          st.i[1] = K;
          st.i[2] = N;
          st.i[3] = 1;  // b stored [n, k]
          st.v = {a, w, n.has_bias ? n.bias : kNone, out};
          st.reads = {a, w};
          if (n.has_bias) st.reads.push_back(n.bias);
          st.writes = {out};
          break;
        }
        if (is_bf16(V(a).dt) && is_bf16(V(w).dt) && is_bf16(V(out).dt) && !n.has_bias &&
            K % 8 == 0 && N % 2 == 0) {
          st.kind = SK::Linear;
          st.bf16 = true;
          st.fmt = sb::WFormat::BF16;
          st.i[0] = M;
          st.i[1] = K;
          st.v = {a, w, kNone, out, kNone};
          st.njobs = 1;
          st.reads = {a, w};
          st.writes = {out};
          break;
        }
        return decline("linear runs as f32, or bf16 without bias");
      }
      case STRATA_OP_RESHAPE: {
        const uint32_t a = in(n, 0);
        if (V(a).bytes() != V(out).bytes())
          fail(STRATA_INVALID_ARGUMENT, "reshape changes the byte size");
        if (is_output[out]) {
          st.kind = SK::Copy;
          st.i[0] = int64_t(V(out).bytes());
          st.v = {a, out};
          st.reads = {a};
          st.writes = {out};
          break;
        }
        exe.alias[out] = exe.alias[a];
        return true;
      }
      case STRATA_OP_TRANSPOSE: {
        const uint32_t a = in(n, 0);
        if (!float_unary_ok(a, out)) return decline("transpose needs f32 or bf16");
        if (V(a).dims.size() != 2 || n.perm != std::vector<int64_t>{1, 0})
          return decline("only the rank-2 [1, 0] transpose is implemented");
        st.kind = SK::Transpose;
        st.bf16 = is_bf16(V(out).dt);
        st.i[0] = V(a).dims[0];
        st.i[1] = V(a).dims[1];
        st.v = {a, out};
        st.reads = {a};
        st.writes = {out};
        break;
      }
      case STRATA_OP_EXPAND: {
        const uint32_t a = in(n, 0);
        if (!float_unary_ok(a, out)) return decline("expand needs f32 or bf16");
        st.kind = SK::Broadcast;
        st.bf16 = is_bf16(V(out).dt);
        if (!bcast(V(out).dims, a, kNone, st.bs)) return decline("operand does not broadcast");
        st.v = {a, out};
        st.reads = {a};
        st.writes = {out};
        break;
      }
      case STRATA_OP_SLICE: {
        const uint32_t a = in(n, 0);
        if (!float_unary_ok(a, out)) return decline("slice needs f32 or bf16");
        if (V(a).dims.size() != 2 || !(n.axis == 1 || n.axis == -1))
          return decline("slice is implemented along axis 1 of a rank-2 tensor");
        if (n.s_stride <= 0) fail(STRATA_INVALID_ARGUMENT, "slice stride must be positive");
        const int64_t cols = V(a).dims[1];
        int64_t cnt = 0, first = -1;
        for (int64_t c = n.s_start; c < n.s_end; c += n.s_stride)
          if (c >= 0 && c < cols) {
            if (first < 0) first = c;
            ++cnt;
          }
        if (V(out).dims != std::vector<int64_t>{V(a).dims[0], cnt})
          fail(STRATA_INVALID_ARGUMENT, "slice output shape does not match its bounds");
        st.kind = SK::Slice;
        st.bf16 = is_bf16(V(out).dt);
        st.i[0] = V(a).dims[0];
        st.i[1] = cols;
        st.i[2] = first < 0 ? 0 : first;
        st.i[3] = n.s_stride;
        st.i[4] = cnt;
        st.v = {a, out};
        st.reads = {a};
        st.writes = {out};
        break;
      }
      case STRATA_OP_CUSTOM:
        return lower_custom(ni);
      default:
        return decline("op tag " + std::to_string(n.op) + " has no kernel");
    }
    push(std::move(st));
    return true;
  }

  bool lower_custom(int ni) {
    const Node& n = g.nodes[ni];
    const std::string& p = n.pattern;
    if (is_linear(n)) return lower_linear(ni);
    const uint32_t out = n.outputs.empty() ? kNone : n.outputs[0];
    Step st;
    st.label = n.name;
    if (p == "fused::rms_norm") {
      const uint32_t x = in(n, 0), gm = in(n, 1);
      if (!float_unary_ok(x, out) || !(V(gm).dt == V(x).dt)) return decline("rms_norm needs matching f32 or bf16");
      if (V(gm).elements() != last_dim(V(x)))
        fail(STRATA_INVALID_ARGUMENT, "rms_norm gamma does not match the trailing axis");
      st.kind = SK::RmsNorm;
      st.bf16 = is_bf16(V(x).dt);
      st.i[0] = rows_of(V(x));
      st.i[1] = last_dim(V(x));
      st.d = n.attr_float("eps", 1e-5);
      st.i[2] = V(gm).producer < 0 ? 1 : 0;  // gamma is a graph input: read before the wait
      st.v = {x, gm, out};
      st.reads = {x, gm};
      st.writes = {out};
    } else if (p == "fused::rope") {
      const uint32_t x = in(n, 0), pos = in(n, 1);
      if (!float_unary_ok(x, out) || !is_i32(V(pos).dt)) return decline("rope needs f32/bf16 x and I32 positions");
      const int64_t hd = n.attr_int("head_dim", 0);
      if (hd <= 0 || hd % 2 || last_dim(V(x)) % hd)
        fail(STRATA_INVALID_ARGUMENT, "rope head_dim must be even and divide the row width");
      if (V(pos).elements() != rows_of(V(x)))
        fail(STRATA_INVALID_ARGUMENT, "rope needs one position per row");
      st.kind = SK::Rope;
      st.bf16 = is_bf16(V(x).dt);
      st.i[0] = rows_of(V(x));
      st.i[1] = last_dim(V(x)) / hd;
      st.i[2] = hd;
      st.d = n.attr_float("theta", 10000.0);
      st.const_off = rope_table(st.d, hd);
      st.v = {x, pos, out};
      st.reads = {x, pos};
      st.writes = {out};
    } else if (p == "fused::swiglu") {
      const uint32_t a = in(n, 0), b = in(n, 1);
      if (!float_unary_ok(a, out) || !(V(b).dt == V(a).dt) || !same_dims(a, b) || !same_dims(a, out))
        return decline("swiglu needs two same-shaped f32 or bf16 operands");
      st.kind = SK::SwiGLU;
      st.bf16 = is_bf16(V(a).dt);
      st.i[0] = V(a).elements();
      st.v = {a, b, out};
      st.reads = {a, b};
      st.writes = {out};
    } else if (p == "fused::attention") {
      const uint32_t q = in(n, 0), k = in(n, 1), v = in(n, 2), kc = in(n, 3), vc = in(n, 4),
                     pos = in(n, 5);
      const DType& dt = V(q).dt;
      if (!is_float(dt) || !(V(k).dt == dt) || !(V(v).dt == dt) || !(V(kc).dt == dt) ||
          !(V(vc).dt == dt) || !(V(out).dt == dt) || !is_i32(V(pos).dt))
        return decline("attention needs one float dtype throughout and I32 positions");
      if (V(kc).dims.size() != 4 || V(kc).dims != V(vc).dims)
        fail(STRATA_INVALID_ARGUMENT, "kv caches must be [batch, kv_heads, max_len, head_dim]");
      // Paged caches (attribute page_size > 0): the caches are page pools
      // [num_pages, kv_heads, page_size, head_dim] and input 6 is the block
      // table I32 [batch, pages_per_seq]; a sequence's max_len is
      // pages_per_seq * page_size.
      const int64_t ps = n.attr_int("page_size", 0);
      uint32_t table = kNone;
      int64_t B = V(kc).dims[0], L = V(kc).dims[2], pps = 0, npages = 0;
      const int64_t KVH = V(kc).dims[1], D = V(kc).dims[3];
      if (ps != 0) {
        if (n.inputs.size() < 7) fail(STRATA_INVALID_ARGUMENT, "paged attention needs a block table (input 6)");
        table = in(n, 6);
        if (!is_i32(V(table).dt) || V(table).dims.size() != 2)
          fail(STRATA_INVALID_ARGUMENT, "the block table must be I32 [batch, pages_per_seq]");
        if (!sb::kv_page_size_ok(ps) || L != ps)
          fail(STRATA_INVALID_ARGUMENT, "page_size must be a power of two from 16 to 4096 and the pages' length");
        if (!is_bf16(dt)) return decline("paged attention runs on bf16 caches only");
        npages = V(kc).dims[0];
        B = V(table).dims[0];
        pps = V(table).dims[1];
        L = pps * ps;
        if (npages <= 0 || pps <= 0 || L > INT32_MAX || npages * KVH * ps > INT32_MAX)
          fail(STRATA_INVALID_ARGUMENT, "paged attention pool or table is empty or too large");
      }
      const int64_t H = n.attr_int("num_heads", 0);
      if (n.attr_int("num_kv_heads", KVH) != KVH || n.attr_int("head_dim", D) != D)
        fail(STRATA_INVALID_ARGUMENT, "attention attributes disagree with the cache shape");
      const int64_t rows = rows_of(V(q));
      if (H <= 0 || last_dim(V(q)) != H * D || last_dim(V(k)) != KVH * D || rows_of(V(k)) != rows ||
          !same_dims(k, v) || !same_dims(q, out) || V(pos).elements() != rows || B <= 0 ||
          rows % B || H % KVH)
        fail(STRATA_INVALID_ARGUMENT, "attention operand shapes are inconsistent");
      if (D != 64 && D != 128) return decline("attention head_dim must be 64 or 128");
      if (H / KVH > 8) return decline("at most 8 query heads per kv head");
      Step ap;
      ap.kind = SK::KvAppend;
      ap.bf16 = is_bf16(dt);
      ap.label = n.name + ".append";
      ap.i[0] = rows;
      ap.i[1] = rows / B;
      ap.i[2] = KVH;
      ap.i[3] = D;
      ap.i[4] = L;
      ap.i[7] = ps;
      ap.i[8] = pps;
      ap.i[9] = npages;
      ap.v = {k, v, kc, vc, pos};
      ap.reads = {k, v, kc, vc, pos};
      ap.writes = {kc, vc};
      if (table != kNone) {
        ap.v.push_back(table);
        ap.reads.push_back(table);
      }
      push(std::move(ap));
      st.kind = SK::Attention;
      st.bf16 = is_bf16(dt);
      st.i[0] = rows;
      st.i[1] = rows / B;
      st.i[2] = H;
      st.i[3] = KVH;
      st.i[4] = D;
      st.i[5] = L;
      // Positions from the host and one token per sequence: cache rows below
      // the position were written by earlier steps, so the attention kernel may
      // stream them before the previous kernel finishes.  With several tokens
      // per sequence this step's own append writes those rows.
      st.i[6] = V(pos).producer < 0 && rows / B == 1 && (table == kNone || V(table).producer < 0) ? 1 : 0;
      st.i[7] = ps;
      st.i[8] = pps;
      st.i[9] = npages;
      st.scratch_bytes = is_bf16(dt) ? sb::attention_v2_scratch_bytes(rows, H, KVH, D, L)
                                     : sb::attention_scratch_bytes(rows, H, KVH, D, L);
      st.v = {q, kc, vc, pos, out};
      st.reads = {q, kc, vc, pos};
      st.writes = {out};
      if (table != kNone) {
        st.v.push_back(table);
        st.reads.push_back(table);
      }
    } else if (p == "fused::embed") {
      const uint32_t ids = in(n, 0), tab = in(n, 1);
      if (!is_i32(V(ids).dt) || !is_float(V(tab).dt) || !(V(out).dt == V(tab).dt) ||
          V(tab).dims.size() != 2)
        return decline("embed needs I32 ids and a rank-2 float table");
      if (last_dim(V(out)) != V(tab).dims[1] || rows_of(V(out)) != V(ids).elements())
        fail(STRATA_INVALID_ARGUMENT, "embed output shape does not match ids x table width");
      st.kind = SK::Embed;
      st.bf16 = is_bf16(V(tab).dt);
      st.i[0] = V(ids).elements();
      st.i[1] = V(tab).dims[0];
      st.i[2] = V(tab).dims[1];
      st.v = {ids, tab, out};
      st.reads = {ids, tab};
      st.writes = {out};
    } else if (p == "fused::argmax") {
      const uint32_t x = in(n, 0);
      if (!is_float(V(x).dt) || !is_i32(V(out).dt)) return decline("argmax maps f32/bf16 rows to I32");
      if (V(out).elements() != rows_of(V(x)))
        fail(STRATA_INVALID_ARGUMENT, "argmax output must have one id per row");
      st.kind = SK::Argmax;
      st.bf16 = is_bf16(V(x).dt);
      st.i[0] = rows_of(V(x));
      st.i[1] = last_dim(V(x));
      st.v = {x, out};
      st.reads = {x};
      st.writes = {out};
    } else if (p == "fused::vocab_argmax") {
      // This rank's lm_head shard's logits [rows, cols]; column c is
      // vocabulary id vocab_offset + c.  Output: the global argmax per row.
      const uint32_t x = in(n, 0);
      if (!is_float(V(x).dt) || !is_i32(V(out).dt)) return decline("vocab_argmax maps f32/bf16 rows to I32");
      if (V(out).elements() != rows_of(V(x)))
        fail(STRATA_INVALID_ARGUMENT, "vocab_argmax output must have one id per row");
      const int64_t off = n.attr_int("vocab_offset", 0);
      if (off < 0 || off + last_dim(V(x)) > int64_t(UINT32_MAX))
        fail(STRATA_INVALID_ARGUMENT, "vocab_argmax vocab_offset is out of range");
      st.kind = SK::VocabArgmax;
      st.bf16 = is_bf16(V(x).dt);
      st.i[0] = rows_of(V(x));
      st.i[1] = last_dim(V(x));
      st.i[2] = off;
      st.scratch_bytes = uint64_t(st.i[0]) * sizeof(uint64_t);  // keys, for the NCCL path
      st.v = {x, out};
      st.reads = {x};
      st.writes = {out};
    } else if (p == "fused::last_token") {
      const uint32_t x = in(n, 0);
      if (!float_unary_ok(x, out)) return decline("last_token needs f32 or bf16");
      const int64_t R = rows_of(V(x)), B = rows_of(V(out));
      if (B <= 0 || R % B || last_dim(V(x)) != last_dim(V(out)) ||
          n.attr_int("tokens_per_seq", R / B) != R / B)
        fail(STRATA_INVALID_ARGUMENT, "last_token maps [batch * tokens, C] to [batch, C]");
      st.kind = SK::LastToken;
      st.bf16 = is_bf16(V(x).dt);
      st.i[0] = B;
      st.i[1] = R / B;
      st.i[2] = last_dim(V(x));
      st.v = {x, out};
      st.reads = {x};
      st.writes = {out};
    } else if (p == "fused::all_reduce") {
      const uint32_t x = in(n, 0);
      if (!float_unary_ok(x, out) || !same_dims(x, out)) return decline("all_reduce needs f32 or bf16");
      if (lower_allreduce_add_norm(ni)) return true;
      st.kind = SK::AllReduce;
      st.bf16 = is_bf16(V(x).dt);
      st.i[0] = V(x).elements();
      st.v = {x, out};
      st.reads = {x};
      st.writes = {out};
    } else if (p == "fused::quantize_w4g32" || p == "fused::quantize_w8pc") {
      const uint32_t w = in(n, 0);
      const bool w4 = p == "fused::quantize_w4g32";
      if (n.outputs.size() != 2 || !is_f32(V(w).dt) || V(w).dims.size() != 2)
        return decline("quantize takes an f32 [N, K] weight and returns (codes, scales)");
      const int64_t N = V(w).dims[0], K = V(w).dims[1];
      const uint32_t c = n.outputs[0], s = n.outputs[1];
      if (w4 ? (!is_w4(V(c).dt) || V(c).dims != std::vector<int64_t>{N, K / 2} || K % 32 ||
                !is_bf16(V(s).dt) || V(s).dims != std::vector<int64_t>{N, K / 32})
             : (!is_w8(V(c).dt) || V(c).dims != std::vector<int64_t>{N, K} || !is_f32(V(s).dt) ||
                V(s).dims != std::vector<int64_t>{N}))
        fail(STRATA_INVALID_ARGUMENT, "quantize output dtypes or shapes are wrong");
      st.kind = w4 ? SK::Quant4 : SK::Quant8;
      st.i[0] = N;
      st.i[1] = K;
      st.v = {w, c, s};
      st.reads = {w};
      st.writes = {c, s};
    } else if (p == "fused::dequantize_w4g32" || p == "fused::dequantize_w8pc") {
      const uint32_t c = in(n, 0), s = in(n, 1);
      const bool w4 = p == "fused::dequantize_w4g32";
      if (!is_f32(V(out).dt) || V(out).dims.size() != 2) return decline("dequantize returns f32 [N, K]");
      const int64_t N = V(out).dims[0], K = V(out).dims[1];
      if (w4 ? (!is_w4(V(c).dt) || V(c).dims != std::vector<int64_t>{N, K / 2} || K % 32 ||
                !is_bf16(V(s).dt) || V(s).dims != std::vector<int64_t>{N, K / 32})
             : (!is_w8(V(c).dt) || V(c).dims != std::vector<int64_t>{N, K} || !is_f32(V(s).dt) ||
                V(s).dims != std::vector<int64_t>{N}))
        fail(STRATA_INVALID_ARGUMENT, "dequantize operand dtypes or shapes are wrong");
      st.kind = w4 ? SK::Dequant4 : SK::Dequant8;
      st.i[0] = N;
      st.i[1] = K;
      st.v = {c, s, out};
      st.reads = {c, s};
      st.writes = {out};
    } else {
      return decline("no kernel for pattern `" + p + "`");
    }
    push(std::move(st));
    return true;
  }
};

// First-fit workspace planner over step-indexed lifetimes.
void plan_workspace(Exe& exe) {
  const Graph& g = exe.g;
  const size_t nv = g.values.size();
  std::vector<int> def(nv, -1), last(nv, -1);
  exe.is_output.assign(nv, false);
  for (auto o : g.outputs) exe.is_output[o] = true;
  exe.needed_input.assign(nv, false);
  for (size_t s = 0; s < exe.steps.size(); ++s) {
    for (auto v : exe.steps[s].reads) {
      const uint32_t b = exe.alias[v];
      last[b] = std::max(last[b], int(s));
      if (g.values[b].producer < 0) exe.needed_input[b] = true;
    }
    for (auto v : exe.steps[s].writes) {
      const uint32_t b = exe.alias[v];
      if (g.values[b].producer >= 0 && def[b] < 0) def[b] = int(s);
      last[b] = std::max(last[b], int(s));
    }
  }
  // Inputs produced by Input nodes are external too.
  for (size_t v = 0; v < nv; ++v) {
    const int64_t p = g.values[v].producer;
    if (p >= 0 && g.nodes[size_t(p)].op == STRATA_OP_INPUT && last[v] >= 0) exe.needed_input[v] = true;
  }
  const int end = int(exe.steps.size());
  for (auto o : g.outputs) {
    const uint32_t b = exe.alias[o];
    if (def[b] >= 0) last[b] = end;
  }
  exe.ws_off.assign(nv, -1);
  struct Block {
    uint64_t off, size;
  };
  std::vector<Block> free_list;
  uint64_t top = 0;
  auto align = [](uint64_t x) { return (x + 255) & ~uint64_t(255); };
  auto alloc = [&](uint64_t size) {
    size = align(std::max<uint64_t>(size, 1));
    for (size_t i = 0; i < free_list.size(); ++i) {
      if (free_list[i].size >= size) {
        const uint64_t off = free_list[i].off;
        free_list[i].off += size;
        free_list[i].size -= size;
        if (free_list[i].size == 0) free_list.erase(free_list.begin() + long(i));
        return off;
      }
    }
    const uint64_t off = top;
    top += size;
    return off;
  };
  auto release = [&](uint64_t off, uint64_t size) {
    size = align(std::max<uint64_t>(size, 1));
    free_list.push_back({off, size});
    std::sort(free_list.begin(), free_list.end(), [](const Block& a, const Block& b) { return a.off < b.off; });
    std::vector<Block> merged;
    for (auto& b : free_list) {
      if (!merged.empty() && merged.back().off + merged.back().size == b.off) merged.back().size += b.size;
      else merged.push_back(b);
    }
    free_list.swap(merged);
  };
  std::vector<std::vector<uint32_t>> dying(exe.steps.size() + 1);
  for (size_t v = 0; v < nv; ++v)
    if (def[v] >= 0) dying[size_t(last[v])].push_back(uint32_t(v));
  for (size_t s = 0; s < exe.steps.size(); ++s) {
    for (auto v : exe.steps[s].writes) {
      const uint32_t b = exe.alias[v];
      if (def[b] == int(s) && exe.ws_off[b] < 0) exe.ws_off[b] = int64_t(alloc(g.values[b].bytes()));
    }
    if (exe.steps[s].scratch_bytes) exe.steps[s].scratch_off = alloc(exe.steps[s].scratch_bytes);
    if (exe.steps[s].scratch_bytes) release(exe.steps[s].scratch_off, exe.steps[s].scratch_bytes);
    for (auto v : dying[s]) release(uint64_t(exe.ws_off[v]), g.values[v].bytes());
  }
  exe.consts_off = (top + 255) / 256 * 256;
  exe.ws_bytes = exe.consts.empty() ? top : exe.consts_off + exe.consts.size();
}

}  // namespace

bool lower(const Graph& g, Exe& exe, std::string* reason) {
  Lowerer L(g, exe, reason);
  if (!L.lower_all()) return false;
  plan_workspace(exe);
  return true;
}

Exe::~Exe() {
  for (auto& c : graphs)
    if (c.exec) cudaGraphExecDestroy(c.exec);
  if (ws) cudaFree(ws);
}

namespace {

struct Ptrs {
  const Exe& exe;
  const std::vector<void*>& ext;
  void* at(uint32_t v) const {
    if (v == kNone) return nullptr;
    const uint32_t b = exe.alias[v];
    if (ext[b]) return ext[b];
    if (exe.ws_off[b] >= 0) return static_cast<char*>(exe.ws) + exe.ws_off[b];
    return nullptr;
  }
};

template <typename T>
T* P(const Ptrs& p, uint32_t v) {
  return static_cast<T*>(p.at(v));
}

// A step's table among the executable's constants, or null.
template <typename T>
const T* const_table(const Exe& exe, const Step& st) {
  if (st.const_off == UINT64_MAX || !exe.ws) return nullptr;
  return reinterpret_cast<const T*>(static_cast<const char*>(exe.ws) + exe.consts_off + st.const_off);
}

// The paged-cache descriptor of an append, attention or fused q/k/v step
// (i[7] page size, i[8] pages per sequence, i[9] pages; the table is operand
// `vi`), or the contiguous default.
sb::KvPages pages_of(const Ptrs& p, const Step& st, size_t vi) {
  sb::KvPages kp;
  if (st.i[7] > 0 && vi < st.v.size()) {
    kp.table = P<const int32_t>(p, st.v[vi]);
    kp.page_size = int(st.i[7]);
    kp.pages_per_seq = int(st.i[8]);
    kp.num_pages = int(st.i[9]);
  }
  return kp;
}

void check_rc(int rc, const Step& st) {
  if (rc == 0) return;
  fail(rc == SB_INVALID_ARGUMENT ? STRATA_INVALID_ARGUMENT : STRATA_INTERNAL,
       "kernel launch for `" + st.label + "` failed (status " + std::to_string(rc) + ")");
}

template <typename T>
int run_float(Ctx& ctx, const Step& st, const Ptrs& p) {
  cudaStream_t s = ctx.stream;
  switch (st.kind) {
    case SK::Binary:
      return sb::launch_binary<T>(int(st.i[0]), P<T>(p, st.v[0]), P<T>(p, st.v[1]), P<T>(p, st.v[2]), st.bs, s);
    case SK::Unary:
      return sb::launch_unary<T>(int(st.i[0]), P<T>(p, st.v[0]), st.i[1], P<T>(p, st.v[1]), s);
    case SK::Softmax:
      return sb::launch_softmax<T>(P<T>(p, st.v[0]), st.i[0], st.i[1], P<T>(p, st.v[1]), s);
    case SK::LayerNorm:
      return sb::launch_layer_norm<T>(P<T>(p, st.v[0]), P<T>(p, st.v[1]), P<T>(p, st.v[2]), st.i[0],
                                      st.i[1], float(st.d), P<T>(p, st.v[3]), s);
    case SK::RmsNorm:
      return sb::launch_rms_norm<T>(P<T>(p, st.v[0]), P<T>(p, st.v[1]), st.i[0], st.i[1], float(st.d),
                                    P<T>(p, st.v[2]), s, st.i[2] != 0);
    case SK::Rope:
      return sb::launch_rope<T>(P<T>(p, st.v[0]), P<int32_t>(p, st.v[1]), st.i[0], st.i[1], st.i[2], st.d,
                                P<T>(p, st.v[2]), s, const_table<double>(p.exe, st));
    case SK::SwiGLU:
      return sb::launch_swiglu<T>(P<T>(p, st.v[0]), P<T>(p, st.v[1]), st.i[0], P<T>(p, st.v[2]), s);
    case SK::Transpose:
      return sb::launch_transpose2<T>(P<T>(p, st.v[0]), st.i[0], st.i[1], P<T>(p, st.v[1]), s);
    case SK::Slice:
      return sb::launch_slice_cols<T>(P<T>(p, st.v[0]), st.i[0], st.i[1], st.i[2], st.i[3], st.i[4],
                                      P<T>(p, st.v[1]), s);
    case SK::Broadcast:
      return sb::launch_broadcast<T>(P<T>(p, st.v[0]), P<T>(p, st.v[1]), st.bs, s);
    case SK::Embed:
      return sb::launch_embed<T>(P<int32_t>(p, st.v[0]), st.i[0], P<T>(p, st.v[1]), st.i[1], st.i[2],
                                 P<T>(p, st.v[2]), ctx.d_err, s);
    case SK::Argmax:
      return sb::launch_argmax<T>(P<T>(p, st.v[0]), st.i[0], st.i[1], P<int32_t>(p, st.v[1]), s);
    case SK::LastToken:
      return sb::launch_last_rows<T>(P<T>(p, st.v[0]), st.i[0], st.i[1], st.i[2], P<T>(p, st.v[1]), s);
    case SK::KvAppend:
      return sb::launch_kv_append<T>(P<T>(p, st.v[0]), P<T>(p, st.v[1]), P<T>(p, st.v[2]), P<T>(p, st.v[3]),
                                     P<int32_t>(p, st.v[4]), st.i[0], st.i[1], st.i[2], st.i[3], st.i[4],
                                     ctx.d_err, s, pages_of(p, st, 5));
    case SK::Attention: {
      float* scratch = st.scratch_bytes ? reinterpret_cast<float*>(static_cast<char*>(p.exe.ws) + st.scratch_off)
                                        : nullptr;
      if constexpr (std::is_same<T, uint16_t>::value)
        return sb::launch_attention_v2(P<T>(p, st.v[0]), P<T>(p, st.v[1]), P<T>(p, st.v[2]),
                                       P<int32_t>(p, st.v[3]), st.i[0], st.i[1], st.i[2], st.i[3], st.i[4],
                                       st.i[5], st.i[6] != 0, scratch, P<T>(p, st.v[4]), ctx.d_err, s,
                                       pages_of(p, st, 5));
      return sb::launch_attention<T>(P<T>(p, st.v[0]), P<T>(p, st.v[1]), P<T>(p, st.v[2]),
                                     P<int32_t>(p, st.v[3]), st.i[0], st.i[1], st.i[2], st.i[3], st.i[4],
                                     st.i[5], scratch, P<T>(p, st.v[4]), ctx.d_err, s);
    }
    default:
      return SB_INTERNAL;
  }
}

// A prefill-sized Linear step: per job, expand the weights to bf16 in the
// step's scratch and run the tcgen05 GEMM (int8 scales in its epilogue); a
// SwiGLU pair expands gate and up side by side and runs one GEMM whose
// epilogue writes silu(gate) * up.
int enqueue_gemm(Ctx& ctx, Exe& exe, const Step& st, const sb::LinearBatch& b, cudaStream_t s) {
  char* base = static_cast<char*>(exe.ws) + st.scratch_off;
  uint64_t wmax = 0;
  for (int j = 0; j < b.njobs; ++j) wmax = std::max<uint64_t>(wmax, uint64_t(b.jobs[j].n) * uint64_t(b.k) * 2);
  const uint64_t wslot = (wmax + 255) / 256 * 256;
  const int fmt = b.fmt == sb::WFormat::W8PC ? 1 : b.fmt == sb::WFormat::MXFP8 ? 2 : b.fmt == sb::WFormat::MXFP4 ? 3 : 0;
  auto scale_of = [&](const sb::LinearJob& J) {
    return b.fmt == sb::WFormat::W8PC ? static_cast<const float*>(J.s) : nullptr;
  };
  if (st.epi == sb::Epilogue::SwiGLU) {
    const sb::LinearJob &G = b.jobs[0], &U = b.jobs[1];
    uint16_t* wg = reinterpret_cast<uint16_t*>(base);
    uint16_t* wu = reinterpret_cast<uint16_t*>(base + wslot);
    if (!sb::gemm_tc_supported(b.m, G.n, b.k, b.x, wg))
      fail(STRATA_INTERNAL, "linear `" + st.label + "` has a layout the tensor-core GEMM cannot take");
    int rc = sb::launch_codes_to_bf16(G.w, G.s, fmt, G.n, b.k, wg, s);
    if (!rc) rc = sb::launch_codes_to_bf16(U.w, U.s, fmt, U.n, b.k, wu, s);
    if (!rc)
      rc = sb::launch_gemm_tc_swiglu(b.x, b.m, b.k, wg, wu, G.n, scale_of(G), scale_of(U), G.y, G.ldy, ctx.d_err, s);
    return rc;
  }
  uint16_t* wbf = reinterpret_cast<uint16_t*>(base);
  for (int j = 0; j < b.njobs; ++j) {
    const sb::LinearJob& J = b.jobs[j];
    if (!J.y) continue;
    if (!sb::gemm_tc_supported(b.m, J.n, b.k, b.x, wbf))
      fail(STRATA_INTERNAL, "linear `" + st.label + "` has a layout the tensor-core GEMM cannot take");
    int rc = sb::launch_codes_to_bf16(J.w, J.s, fmt, J.n, b.k, wbf, s);
    if (rc) return rc;
    rc = sb::launch_gemm_tc_bf16(b.x, b.m, b.k, wbf, J.n, scale_of(J), J.residual, J.ldr, J.y, J.ldy, ctx.d_err, s);
    if (rc) return rc;
  }
  return SB_OK;
}

}  // namespace

namespace {

// The class a step's device time is reported under.
const char* step_class(const Step& st) {
  switch (st.kind) {
    case SK::Linear:
      if (st.scratch_bytes) return st.epi == sb::Epilogue::SwiGLU ? "gemm:swiglu" : "gemm";
      return st.epi == sb::Epilogue::SwiGLU ? "gemv:swiglu" : st.epi == sb::Epilogue::Residual ? "gemv:residual" : "gemv";
    case SK::QkvRope: return "gemv:qkv_rope_append";
    case SK::Attention: return "attention";
    case SK::KvAppend: return "kv_append";
    case SK::AllReduce: return "all_reduce";
    case SK::AllReduceAddNorm: return "all_reduce_add_norm";
    case SK::RmsNorm: return "rms_norm";
    case SK::Rope: return "rope";
    case SK::Embed: return "embed";
    case SK::Argmax: return "argmax";
    case SK::VocabArgmax: return "vocab_argmax";
    case SK::LastToken: return "last_token";
    case SK::Binary: return "add_mul";
    default: return "other";
  }
}

void ev_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) fail(STRATA_INTERNAL, std::string(what) + ": " + cudaGetErrorString(e));
}

struct StepClock {
  std::mutex mu;
  std::map<std::string, std::pair<uint64_t, double>> acc;  // class -> (steps, ms)
};

StepClock& step_clock() {
  static StepClock c;
  return c;
}

// Events around every step of one eager run; destroyed on every path.
struct StepEvents {
  std::vector<cudaEvent_t> ev;
  explicit StepEvents(size_t n) : ev(n, nullptr) {
    for (auto& e : ev) ev_check(cudaEventCreate(&e), "cudaEventCreate");
  }
  ~StepEvents() {
    for (auto e : ev)
      if (e) cudaEventDestroy(e);
  }
};

}  // namespace

bool step_times_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("STRATA_B200_STEP_TIMES");
    return v && *v && *v != '0';
  }();
  return on;
}

std::string step_times_json(bool reset) {
  StepClock& c = step_clock();
  std::lock_guard<std::mutex> lk(c.mu);
  std::string out = "{";
  char buf[96];
  bool first = true;
  for (const auto& kv : c.acc) {
    std::snprintf(buf, sizeof(buf), "%s\"%s\": [%llu, %.6f]", first ? "" : ", ", kv.first.c_str(),
                  static_cast<unsigned long long>(kv.second.first), kv.second.second);
    out += buf;
    first = false;
  }
  out += "}";
  if (reset) c.acc.clear();
  return out;
}

namespace {

void enqueue_steps(Ctx& ctx, Exe& exe, const std::vector<void*>& ext, StepEvents* events);

}  // namespace

void enqueue(Ctx& ctx, Exe& exe, const std::vector<void*>& ext) {
  if (!step_times_enabled()) {
    enqueue_steps(ctx, exe, ext, nullptr);
    return;
  }
  StepEvents events(exe.steps.size() + 1);
  ev_check(cudaEventRecord(events.ev[0], ctx.stream), "cudaEventRecord");
  enqueue_steps(ctx, exe, ext, &events);
  ev_check(cudaEventSynchronize(events.ev.back()), "cudaEventSynchronize");
  StepClock& c = step_clock();
  std::lock_guard<std::mutex> lk(c.mu);
  for (size_t i = 0; i < exe.steps.size(); ++i) {
    float ms = 0.0f;
    ev_check(cudaEventElapsedTime(&ms, events.ev[i], events.ev[i + 1]), "cudaEventElapsedTime");
    auto& a = c.acc[step_class(exe.steps[i])];
    a.first += 1;
    a.second += double(ms);
  }
}

namespace {

void enqueue_steps(Ctx& ctx, Exe& exe, const std::vector<void*>& ext, StepEvents* events) {
  Ptrs p{exe, ext};
  cudaStream_t s = ctx.stream;
  size_t si = 0;
  for (const Step& st : exe.steps) {
    int rc = 0;
    switch (st.kind) {
      case SK::Linear: {
        sb::LinearBatch b{};
        b.x = P<uint16_t>(p, st.v[0]);
        b.m = int(st.i[0]);
        b.k = int(st.i[1]);
        b.fmt = st.fmt;
        b.epi = st.epi;
        b.njobs = st.njobs;
        for (int j = 0; j < st.njobs; ++j) {
          const uint32_t w = st.v[1 + 4 * j], sc = st.v[2 + 4 * j], y = st.v[3 + 4 * j], r = st.v[4 + 4 * j];
          const Value& wv = exe.g.values[w];
          const int n = int(wv.dims[0]);
          b.jobs[j] = sb::LinearJob{p.at(w), p.at(sc), n, P<uint16_t>(p, y), n, P<uint16_t>(p, r), n};
        }
        if (st.scratch_bytes) {
          rc = enqueue_gemm(ctx, exe, st, b, s);
          break;
        }
        sb::GemvMmaArgs ga{};
        ga.lb = b;
        ga.mode = st.epi == sb::Epilogue::SwiGLU ? sb::GemvMode::SwiGLU : sb::GemvMode::Plain;
        ga.pdl = sb::pdl_enabled();
        rc = sb::gemv_mma_supported(ga) ? sb::launch_gemv_mma(ga, s) : sb::launch_linear(b, s);
        break;
      }
      case SK::QkvRope: {
        sb::GemvMmaArgs ga{};
        sb::LinearBatch& b = ga.lb;
        b.x = P<uint16_t>(p, st.v[0]);
        b.m = int(st.i[0]);
        b.k = int(st.i[1]);
        b.fmt = st.fmt;
        b.epi = sb::Epilogue::None;
        b.njobs = 3;
        const int hd = int(st.i[4]);
        const int ns[3] = {int(st.i[2]) * hd, int(st.i[3]) * hd, int(st.i[3]) * hd};
        for (int j = 0; j < 3; ++j)
          b.jobs[j] = sb::LinearJob{p.at(st.v[1 + 2 * j]), p.at(st.v[2 + 2 * j]), ns[j], nullptr, ns[j], nullptr, ns[j]};
        ga.mode = sb::GemvMode::QkvRope;
        ga.pdl = sb::pdl_enabled();
        sb::QkvExtra& e = ga.qkv;
        e.pos = P<int32_t>(p, st.v[10]);
        e.q_out = P<uint16_t>(p, st.v[7]);
        e.k_cache = P<uint16_t>(p, st.v[8]);
        e.v_cache = P<uint16_t>(p, st.v[9]);
        e.hq = int(st.i[2]);
        e.hkv = int(st.i[3]);
        e.head_dim = hd;
        e.max_len = int(st.i[5]);
        e.tokens_per_seq = int(st.i[6]);
        e.theta = st.d;
        e.err = ctx.d_err;
        e.kp = pages_of(p, st, 11);
        e.inv_freq = const_table<double>(exe, st);
        if (!sb::gemv_mma_supported(ga))
          fail(STRATA_INTERNAL, "fused q/k/v projection `" + st.label + "` has an unsupported layout");
        rc = sb::launch_gemv_mma(ga, s);
        break;
      }
      case SK::GemmF32:
        rc = sb::launch_gemm_f32(P<float>(p, st.v[0]), P<float>(p, st.v[1]), P<float>(p, st.v[2]), st.i[0],
                                 st.i[1], st.i[2], st.i[3] != 0, P<float>(p, st.v[3]), s);
        break;
      case SK::Copy: {
        void* dst = p.at(st.v[1]);
        const void* src = p.at(st.v[0]);
        if (dst != src && cudaMemcpyAsync(dst, src, size_t(st.i[0]), cudaMemcpyDeviceToDevice, s) != cudaSuccess)
          rc = SB_INTERNAL;
        break;
      }
      case SK::VocabArgmax: {
        const int64_t rows = st.i[0], cols = st.i[1], off = st.i[2];
        int32_t* out = P<int32_t>(p, st.v[1]);
        const void* x = p.at(st.v[0]);
        const bool peer = ctx.world > 1 && ctx.ar_ready && rows <= sb::kAmMaxRows;
        const bool nccl = ctx.world > 1 && !peer && ctx.comm;
        if (ctx.world > 1 && !peer && !nccl)
          fail(STRATA_INTERNAL, "vocab_argmax `" + st.label + "` needs the tensor-parallel communicator");
        uint64_t* keys = nccl ? reinterpret_cast<uint64_t*>(static_cast<char*>(p.exe.ws) + st.scratch_off) : nullptr;
        const int world = ctx.world > 1 ? ctx.world : 1;
        rc = st.bf16 ? sb::launch_vocab_argmax<uint16_t>(static_cast<const uint16_t*>(x), rows, cols, off, ctx.rank,
                                                         world, &ctx.ar_peers, ctx.ar_counters, keys, out, ctx.d_err, s)
                     : sb::launch_vocab_argmax<float>(static_cast<const float*>(x), rows, cols, off, ctx.rank, world,
                                                      &ctx.ar_peers, ctx.ar_counters, keys, out, ctx.d_err, s);
        if (rc == 0 && nccl) {
          const ncclResult_t r = ctx.nccl.all_reduce(keys, keys, size_t(rows), ncclUint64, ncclMax, ctx.comm, s);
          if (r != ncclSuccess)
            fail(STRATA_INTERNAL, std::string("ncclAllReduce failed: ") + ctx.nccl.error_string(r));
          rc = sb::launch_vocab_argmax_decode(keys, rows, out, s);
        }
        break;
      }
      case SK::AllReduce: {
        void* src = p.at(st.v[0]);
        void* dst = p.at(st.v[1]);
        if (ctx.ar_ready && st.bf16 && sb::allreduce_bf16_supported(st.i[0], src, dst, ctx.world)) {
          rc = sb::launch_allreduce_bf16(static_cast<const uint16_t*>(src), static_cast<uint16_t*>(dst), st.i[0],
                                         ctx.rank, ctx.world, ctx.ar_peers, ctx.ar_counters, ctx.d_err, s);
        } else if (ctx.comm && ctx.world > 1) {
          const ncclResult_t r = ctx.nccl.all_reduce(src, dst, size_t(st.i[0]),
                                                     st.bf16 ? ncclBfloat16 : ncclFloat32, ncclSum,
                                                     ctx.comm, s);
          if (r != ncclSuccess)
            fail(STRATA_INTERNAL, std::string("ncclAllReduce failed: ") + ctx.nccl.error_string(r));
        } else if (dst != src) {
          const size_t bytes = size_t(st.i[0]) * (st.bf16 ? 2 : 4);
          if (cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, s) != cudaSuccess) rc = SB_INTERNAL;
        }
        break;
      }
      case SK::AllReduceAddNorm: {
        // v = {x, r, gamma, h, y}: h = all_reduce(x) + r, y = rms_norm(h) * gamma.
        const auto* x = P<uint16_t>(p, st.v[0]);
        const auto* r = P<uint16_t>(p, st.v[1]);
        const auto* gm = P<uint16_t>(p, st.v[2]);
        auto* h = P<uint16_t>(p, st.v[3]);
        auto* y = P<uint16_t>(p, st.v[4]);
        const int64_t rows = st.i[0], cols = st.i[1];
        if (ctx.ar_ready && sb::allreduce_add_norm_supported(rows, cols, x, r, gm, h, y, ctx.world)) {
          rc = sb::launch_allreduce_add_norm_bf16(x, r, gm, h, y, rows, cols, float(st.d), ctx.rank, ctx.world,
                                                  ctx.ar_peers, ctx.ar_counters, ctx.d_err, s);
          break;
        }
        // Otherwise: the sum into y (free until the norm writes it), the add
        // into h, the norm into y.
        const uint16_t* sum = x;
        if (ctx.comm && ctx.world > 1) {
          const ncclResult_t e = ctx.nccl.all_reduce(x, y, size_t(rows * cols), ncclBfloat16, ncclSum, ctx.comm, s);
          if (e != ncclSuccess)
            fail(STRATA_INTERNAL, std::string("ncclAllReduce failed: ") + ctx.nccl.error_string(e));
          sum = y;
        }
        rc = sb::launch_binary<uint16_t>(0, sum, r, h, st.bs, s);
        if (rc == 0) rc = sb::launch_rms_norm<uint16_t>(h, gm, rows, cols, float(st.d), y, s);
        break;
      }
      case SK::Quant4:
        rc = sb::launch_quant_w4g32(P<float>(p, st.v[0]), st.i[0], st.i[1], P<uint8_t>(p, st.v[1]),
                                    P<uint16_t>(p, st.v[2]), s);
        break;
      case SK::Quant8:
        rc = sb::launch_quant_w8pc(P<float>(p, st.v[0]), st.i[0], st.i[1], P<int8_t>(p, st.v[1]),
                                   P<float>(p, st.v[2]), s);
        break;
      case SK::Dequant4:
        rc = sb::launch_dequant_w4g32(P<uint8_t>(p, st.v[0]), P<uint16_t>(p, st.v[1]), st.i[0], st.i[1],
                                      P<float>(p, st.v[2]), s);
        break;
      case SK::Dequant8:
        rc = sb::launch_dequant_w8pc(P<int8_t>(p, st.v[0]), P<float>(p, st.v[1]), st.i[0], st.i[1],
                                     P<float>(p, st.v[2]), s);
        break;
      default:
        rc = st.bf16 ? run_float<uint16_t>(ctx, st, p) : run_float<float>(ctx, st, p);
        break;
    }
    check_rc(rc, st);
    ++si;
    if (events) ev_check(cudaEventRecord(events->ev[si], s), "cudaEventRecord");
  }
}

}  // namespace

}  // namespace sbp
