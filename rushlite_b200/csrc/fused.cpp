// The lazy-fusion compiler: lmpb_fused_build / launch / release.
//
// Takes a DAG of elementwise nodes over one iteration space (see lmpb.h),
// plans it, generates a CUDA C++ kernel, compiles it with NVRTC for sm_100a
// and caches the cubin in memory and on disk.  Compared with the reference
// inductor (csrc/src/inductor/nvrtc/{fused_graph,codegen,nvrtc_backend}.cpp):
//  * leaves may broadcast, so a whole broadcast chain is one kernel;
//  * the iteration space is collapsed (size-1 dims dropped, dims merged where
//    every leaf and output agrees), divisions are by compile-time constants;
//  * each thread handles a VEC-wide packet of the innermost dim with 128-bit
//    loads/stores in a grid-stride loop sized to the SM count; values that do
//    not vary along the packet (row-broadcast leaves and everything computed
//    only from them) are computed once per packet, and once per row in the
//    reduction patterns;
//  * outputs can accumulate into an existing buffer (add_inplace fused) or be
//    summed over broadcast axes (sum_broadcast_axis fused) with a CTA/warp
//    tree per row, or a deterministic split-row column sum;
//  * NVRTC is given --fmad=false and every + - * is an explicit _rn op, so a
//    fused chain rounds like the op-by-op path;
//  * cubins persist on disk keyed by a hash of the source, so a new process
//    does not recompile.
#include <cuda.h>
#include <cuda_runtime.h>
#include <nvrtc.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <array>
#include <cstdint>
#include <fstream>
#include <map>
#include <memory>
#include <mutex>
#include <sstream>
#include <string>
#include <vector>

#include "lmpb.h"
#include "ops_device_inc.h"  // kOpsDeviceSource: ops_device.cuh as a string (generated)

namespace lmpb {
lmpb_status set_error(lmpb_status st, const std::string& msg);
bool valid_dtype(int dt);
size_t dtype_size(int dt);
int sm_count();
void count_launch();
cudaError_t stream_alloc(void** p, size_t bytes, cudaStream_t st);
}  // namespace lmpb

using lmpb::set_error;

namespace {

constexpr int kThreads = 256;

enum Pattern { kElementwise = 0, kRowReduce = 1, kColReduce = 2 };

const char* ctype(int dt) {
  switch (dt) {
    case LMPB_BOOL: return "bool";
    case LMPB_INT16: return "short";
    case LMPB_INT32: return "int";
    case LMPB_INT64: return "long long";
    case LMPB_FLOAT32: return "float";
    default: return "double";
  }
}

std::string dlit(double v) {
  char buf[64];
  snprintf(buf, sizeof buf, "%a", v);  // exact hex-float literal
  std::string s(buf);
  if (s == "inf") return "(1.0/0.0)";
  if (s == "-inf") return "(-1.0/0.0)";
  if (s == "nan" || s == "-nan") return "(0.0/0.0)";
  return s;
}

uint64_t fnv1a(const std::string& s) {
  uint64_t h = 1469598103934665603ull;
  for (unsigned char c : s) {
    h ^= c;
    h *= 1099511628211ull;
  }
  return h;
}

struct Plan {
  Pattern pattern = kElementwise;
  int G = 1;                       // collapsed groups
  std::array<int64_t, LMPB_MAX_DIMS> size{};
  std::vector<std::array<int64_t, LMPB_MAX_DIMS>> leaf_stride;  // per leaf, per group
  std::vector<std::array<int64_t, LMPB_MAX_DIMS>> out_stride;   // per output, per group
  std::vector<int> out_mode;       // STORE/ACCUM or reduce (after normalisation)
  int64_t n = 0;                   // iteration elements
  int vec = 1;                     // packet width of the vector kernel
  bool idx32 = true;
  int64_t S = 1;                   // column-reduce row chunks
  bool warp_rows = false;          // row-reduce: warp per row
  int row_unroll = 1;              // row-reduce: unroll factor of the walk along a row
  int stream = 0;                  // 1: full-size outputs use evict-first stores; 2: leaf loads too
};

}  // namespace

struct lmpb_fused_s {
  std::string source;
  Plan plan;
  std::vector<lmpb_fnode> nodes;
  std::vector<lmpb_fleaf> leaves;
  std::vector<lmpb_fout> outs;
  std::vector<size_t> ws_offset;  // per output (column reduce with S > 1)
  size_t ws_bytes = 0;
  std::mutex mu;
  std::map<CUcontext, std::array<CUfunction, 3>> fn;  // vector, scalar, combine
};

namespace {

// ------------------------------------------------------------------ planning

lmpb_status make_plan(lmpb_fused_s& h, const int64_t* iter, int nd) {
  Plan& p = h.plan;
  const int NL = (int)h.leaves.size(), NO = (int)h.outs.size();
  // per-dim signature: bit per leaf (broadcast) and per output (reduced)
  std::vector<std::vector<char>> sig(nd);
  std::vector<std::vector<int64_t>> lstride(NL, std::vector<int64_t>(nd, 0));
  std::vector<std::vector<int64_t>> ostride(NO, std::vector<int64_t>(nd, 0));
  auto right_align = [&](const int64_t* shape, int snd, std::vector<int64_t>& stride,
                         std::vector<char>& bcast, const char* what) -> lmpb_status {
    if (snd > nd) return set_error(LMPB_ERR_INVALID, std::string("fused: ") + what + " has more dims than the iteration space");
    int64_t s = 1;
    for (int k = 0; k < nd; ++k) {
      const int d = nd - 1 - k;
      const int src = snd - 1 - k;
      const int64_t ext = src >= 0 ? shape[src] : 1;
      if (ext == iter[d]) {
        stride[d] = iter[d] == 1 ? 0 : s;
        bcast[d] = 0;
      } else if (ext == 1) {
        stride[d] = 0;
        bcast[d] = 1;
      } else {
        return set_error(LMPB_ERR_INVALID, std::string("fused: ") + what + " does not broadcast to the iteration space");
      }
      s *= ext;
    }
    return LMPB_OK;
  };
  std::vector<std::vector<char>> lb(NL, std::vector<char>(nd, 0)), ob(NO, std::vector<char>(nd, 0));
  for (int i = 0; i < NL; ++i) {
    lmpb_status st = right_align(h.leaves[i].shape, h.leaves[i].ndim, lstride[i], lb[i], "leaf");
    if (st != LMPB_OK) return st;
  }
  p.out_mode.resize(NO);
  bool any_reduce = false;
  for (int j = 0; j < NO; ++j) {
    lmpb_status st = right_align(h.outs[j].shape, h.outs[j].ndim, ostride[j], ob[j], "output");
    if (st != LMPB_OK) return st;
    int mode = h.outs[j].mode;
    bool reduced = false;
    for (int d = 0; d < nd; ++d) reduced |= ob[j][d] != 0;
    if (mode == LMPB_OUT_STORE || mode == LMPB_OUT_ACCUM) {
      if (reduced) return set_error(LMPB_ERR_INVALID, "fused: STORE/ACCUM output must have the iteration shape");
    } else if (!reduced) {
      mode = mode == LMPB_OUT_REDUCE_SUM ? LMPB_OUT_STORE : LMPB_OUT_ACCUM;
    } else {
      any_reduce = true;
    }
    p.out_mode[j] = mode;
  }
  // in-kernel row reductions reduce the last iteration dim: keep it a group of its own
  bool any_rowred = false;
  for (const auto& n : h.nodes) any_rowred |= n.kind == LMPB_FN_ROWRED;
  if (any_rowred && (nd == 0 || iter[nd - 1] <= 1))
    return set_error(LMPB_ERR_INVALID, "fused: a row reduction needs a last iteration dim longer than 1");
  // collapse
  p.n = 1;
  for (int d = 0; d < nd; ++d) p.n *= iter[d];
  int G = 0;
  std::vector<std::vector<char>> gsig;
  for (int d = 0; d < nd; ++d) {
    if (iter[d] == 1) continue;
    std::vector<char> s;
    for (int i = 0; i < NL; ++i) s.push_back(lb[i][d]);
    for (int j = 0; j < NO; ++j) s.push_back(ob[j][d]);
    s.push_back(any_rowred && d == nd - 1);
    if (G > 0 && gsig[G - 1] == s) {
      p.size[G - 1] *= iter[d];
      for (int i = 0; i < NL; ++i) p.leaf_stride[i][G - 1] = lstride[i][d];
      for (int j = 0; j < NO; ++j) p.out_stride[j][G - 1] = ostride[j][d];
      continue;
    }
    if (G == 0) {
      p.leaf_stride.assign(NL, {});
      p.out_stride.assign(NO, {});
    }
    gsig.push_back(s);
    p.size[G] = iter[d];
    for (int i = 0; i < NL; ++i) p.leaf_stride[i][G] = lstride[i][d];
    for (int j = 0; j < NO; ++j) p.out_stride[j][G] = ostride[j][d];
    ++G;
  }
  if (G == 0) {  // a single element
    p.leaf_stride.assign(NL, {});
    p.out_stride.assign(NO, {});
    p.size[0] = 1;
    G = 1;
  }
  p.G = G;
  p.idx32 = p.n < (1ll << 31);
  // pattern
  if (any_rowred) {
    // one warp or CTA per row (the last dim); reduce outputs may only reduce the row
    if (G == 1) {  // the whole space is one row
      p.G = 2;
      p.size[1] = p.size[0];
      p.size[0] = 1;
      for (auto& s : p.leaf_stride) { s[1] = s[0]; s[0] = 0; }
      for (auto& s : p.out_stride) { s[1] = s[0]; s[0] = 0; }
    } else if (G != 2) {
      return set_error(LMPB_ERR_UNSUPPORTED, "fused: row reductions over a space of more than two groups");
    }
    for (int j = 0; j < NO; ++j) {
      if (p.out_mode[j] < LMPB_OUT_REDUCE_SUM) continue;
      if (p.out_stride[j][0] == 0 && p.size[0] > 1)
        return set_error(LMPB_ERR_UNSUPPORTED, "fused: row reductions with a reduction over rows");
    }
    p.pattern = kRowReduce;
  } else if (any_reduce) {
    std::vector<char> red;
    for (int j = 0; j < NO; ++j) {
      if (p.out_mode[j] != LMPB_OUT_REDUCE_SUM && p.out_mode[j] != LMPB_OUT_REDUCE_SUM_ACCUM) continue;
      std::vector<char> r(G);
      for (int g = 0; g < G; ++g) r[g] = p.out_stride[j][g] == 0 && p.size[g] > 1;
      if (red.empty()) red = r;
      else if (red != r) return set_error(LMPB_ERR_UNSUPPORTED, "fused: outputs reduce over different axes");
    }
    if (G == 2 && !red[0] && red[1]) p.pattern = kRowReduce;
    else if (G == 2 && red[0] && !red[1]) p.pattern = kColReduce;
    else if (G == 1 && red[0]) {  // full reduction of a 1-D space: treat as one row
      p.G = 2;
      p.size[1] = p.size[0];
      p.size[0] = 1;
      for (auto& s : p.leaf_stride) { s[1] = s[0]; s[0] = 0; }
      for (auto& s : p.out_stride) { s[1] = s[0]; s[0] = 0; }
      p.pattern = kRowReduce;
    } else {
      return set_error(LMPB_ERR_UNSUPPORTED, "fused: reduction pattern not supported in one kernel");
    }
  }
  const int64_t inner = p.size[p.G - 1];
  int want = p.pattern == kElementwise ? 4 : 8;  // measured best on B200 (C2 sweep)
  if (const char* e = getenv(p.pattern == kElementwise ? "LMPB_FUSED_VEC_EW" : "LMPB_FUSED_VEC_RED")) {
    const int v = atoi(e);  // tuning override: 1, 2, 4, 8 or 16
    if (v == 1 || v == 2 || v == 4 || v == 8 || v == 16) want = v;
  }
  if (const char* e = getenv("LMPB_FUSED_STREAM")) p.stream = std::max(0, std::min(2, atoi(e)));  // tuning override
  p.vec = 1;
  for (int v = want; v > 1; v >>= 1)
    if (inner % v == 0) { p.vec = v; break; }
  if (p.pattern == kRowReduce) {
    int64_t warp_max = 2048;  // rows shorter than this get a warp each, longer ones a CTA
    if (const char* e = getenv("LMPB_FUSED_WARP_ROWS")) warp_max = atoll(e);  // tuning override
    p.warp_rows = inner < warp_max;
    if (const char* e = getenv("LMPB_FUSED_ROW_UNROLL")) p.row_unroll = std::max(1, atoi(e));  // tuning override
  }
  if (p.pattern == kColReduce) {
    const int64_t Q = p.size[1], P = p.size[0];
    const int64_t colblocks = (Q / p.vec + kThreads - 1) / kThreads;
    const int64_t target = (int64_t)lmpb::sm_count() * 4;
    int64_t S = 1;
    if (colblocks < target && P >= 64) {
      S = (target + colblocks - 1) / colblocks;
      if (S > P / 16) S = P / 16;
      if (S < 1) S = 1;
    }
    p.S = S;
    if (S > 65535) p.S = 65535;
  }
  return LMPB_OK;
}

// -------------------------------------------------------------------- codegen

struct Gen {
  const lmpb_fused_s& h;
  const Plan& p;
  int vec;
  std::ostringstream os;
  std::vector<std::array<bool, LMPB_MAX_DIMS>> varies;  // per node, per group
  std::string I;                                          // index type
  explicit Gen(const lmpb_fused_s& hh, int v) : h(hh), p(hh.plan), vec(v) {
    I = p.idx32 ? "unsigned" : "unsigned long long";
    const int NN = (int)h.nodes.size();
    varies.assign(NN, {});
    for (int m = 0; m < NN; ++m) {
      const lmpb_fnode& nd = h.nodes[m];
      for (int g = 0; g < p.G; ++g) {
        bool v = false;
        if (nd.kind == LMPB_FN_LEAF) v = p.leaf_stride[nd.a][g] != 0;
        else if (nd.kind == LMPB_FN_BINARY) v = varies[nd.a][g] || varies[nd.b][g];
        else if (nd.kind == LMPB_FN_UNARY) v = varies[nd.a][g];
        else if (nd.kind == LMPB_FN_ROWRED) v = g < p.G - 1 && varies[nd.a][g];  // constant along its row
        varies[m][g] = v;
      }
    }
  }
  bool lane(int m) const { return vec > 1 && varies[m][p.G - 1]; }
  std::string ref(int m, bool in_lane_loop) const {
    std::string s = "v" + std::to_string(m);
    if (in_lane_loop && lane(m)) s += "[j]";
    return s;
  }
  std::string tname(int dt) const { return ctype(dt); }

  // Emits the computation of node m; `off` maps a leaf slot to its offset expression.
  void emit_node(int m, const std::string& ind, const std::vector<std::string>& leaf_off) {
    const lmpb_fnode& nd = h.nodes[m];
    if (nd.kind == LMPB_FN_ROWRED) return;  // declared by its walk in gen_row_reduce
    const std::string T = tname(nd.dtype);
    const bool L = lane(m);
    const std::string decl = "    " + ind + T + " v" + std::to_string(m) + (L ? "[" + std::to_string(vec) + "]" : "");
    if (nd.kind == LMPB_FN_CONST) {
      os << decl << " = static_cast<" << T << ">(" << dlit(nd.p0) << ");\n";
      return;
    }
    if (nd.kind == LMPB_FN_LEAF) {
      const std::string src = "L" + std::to_string(nd.a);
      const std::string LT = tname(h.leaves[nd.a].dtype);
      if (L) {
        if (p.stream >= 2 && (vec * (int)lmpb::dtype_size(h.leaves[nd.a].dtype)) % 16 == 0)
          os << "    " << ind << "Pack<" << LT << ", " << vec << "> pk" << m << " = ld_cs<" << LT << ", " << vec << ">("
             << src << " + " << leaf_off[nd.a] << ");\n";
        else
          os << "    " << ind << "Pack<" << LT << ", " << vec << "> pk" << m << " = *reinterpret_cast<const Pack<" << LT
             << ", " << vec << ">*>(" << src << " + " << leaf_off[nd.a] << ");\n";
        os << decl << ";\n";
        os << "    " << ind << "#pragma unroll\n    " << ind << "for (int j = 0; j < " << vec << "; ++j) v" << m
           << "[j] = static_cast<" << T << ">(pk" << m << ".v[j]);\n";
      } else {
        os << decl << " = static_cast<" << T << ">(" << src << "[" << leaf_off[nd.a] << "]);\n";
      }
      return;
    }
    std::string expr;
    const std::string lo = "static_cast<" + T + ">(" + dlit(nd.p0) + ")";
    const std::string hi = "static_cast<" + T + ">(" + dlit(nd.p1) + ")";
    auto in = [&](int k) { return "static_cast<" + T + ">(" + ref(k, true) + ")"; };
    if (nd.kind == LMPB_FN_BINARY)
      expr = "lmpb_dev::binary_apply<" + std::to_string(nd.sub) + ", " + T + ">(" + in(nd.a) + ", " + in(nd.b) + ", " + lo + ", " + hi + ")";
    else
      expr = "lmpb_dev::unary_apply<" + std::to_string(nd.sub) + ", " + T + ">(" + in(nd.a) + ", " + lo + ", " + hi + ")";
    if (L) {
      os << decl << ";\n";
      os << "    " << ind << "#pragma unroll\n    " << ind << "for (int j = 0; j < " << vec << "; ++j) v" << m << "[j] = " << expr << ";\n";
    } else {
      // operands are scalars here; ref(k, true) gives plain names
      os << decl << " = " << expr << ";\n";
    }
  }

  // Emits the full-size STORE/ACCUM outputs at element offset `off` (contiguous).
  void emit_full_outputs(const std::string& ind, const std::string& off) {
    for (size_t j = 0; j < h.outs.size(); ++j) {
      const int mode = p.out_mode[j];
      if (mode != LMPB_OUT_STORE && mode != LMPB_OUT_ACCUM) continue;
      const int m = h.outs[j].node;
      const std::string OT = tname(h.outs[j].dtype);
      const std::string O = "O" + std::to_string(j);
      const bool cs = p.stream >= 1 && (vec * (int)lmpb::dtype_size(h.outs[j].dtype)) % 16 == 0;
      if (vec > 1) {
        os << "    " << ind << "{ Pack<" << OT << ", " << vec << "> po;\n";
        if (mode == LMPB_OUT_ACCUM && cs)
          os << "    " << ind << "  po = ld_cs<" << OT << ", " << vec << ">(" << O << " + " << off << ");\n";
        else if (mode == LMPB_OUT_ACCUM)
          os << "    " << ind << "  po = *reinterpret_cast<const Pack<" << OT << ", " << vec << ">*>(" << O << " + " << off << ");\n";
        os << "    " << ind << "  #pragma unroll\n    " << ind << "  for (int j = 0; j < " << vec << "; ++j) po.v[j] = ";
        if (mode == LMPB_OUT_ACCUM)
          os << "lmpb_dev::r_add<" << OT << ">(po.v[j], static_cast<" << OT << ">(" << ref(m, true) << "));\n";
        else
          os << "static_cast<" << OT << ">(" << ref(m, true) << ");\n";
        if (cs)
          os << "    " << ind << "  st_cs<" << OT << ", " << vec << ">(" << O << " + " << off << ", po); }\n";
        else
          os << "    " << ind << "  *reinterpret_cast<Pack<" << OT << ", " << vec << ">*>(" << O << " + " << off << ") = po; }\n";
      } else {
        if (mode == LMPB_OUT_ACCUM)
          os << "    " << ind << O << "[" << off << "] = lmpb_dev::r_add<" << OT << ">(" << O << "[" << off << "], static_cast<" << OT << ">(" << ref(m, false) << "));\n";
        else
          os << "    " << ind << O << "[" << off << "] = static_cast<" << OT << ">(" << ref(m, false) << ");\n";
      }
    }
  }

  void prologue(const std::string& name) {
    os << "extern \"C\" __global__ void __launch_bounds__(" << kThreads << ") " << name << "(const Params prm) {\n";
    for (size_t i = 0; i < h.leaves.size(); ++i)
      os << "  const " << tname(h.leaves[i].dtype) << "* __restrict__ L" << i << " = static_cast<const "
         << tname(h.leaves[i].dtype) << "*>(prm.leaf[" << i << "]);\n";
    for (size_t j = 0; j < h.outs.size(); ++j)
      os << "  " << tname(h.outs[j].dtype) << "* __restrict__ O" << j << " = static_cast<" << tname(h.outs[j].dtype)
         << "*>(prm.out[" << j << "]);\n";
  }

  std::vector<int> nodes_where(bool (Gen::*pred)(int) const) const {
    std::vector<int> r;
    for (int m = 0; m < (int)h.nodes.size(); ++m)
      if ((this->*pred)(m)) r.push_back(m);
    return r;
  }

  // offset expression of a leaf from group coordinates c0..c(G-1)
  std::string leaf_offset(int i, const std::vector<std::string>& coord) const {
    std::string s;
    for (int g = 0; g < p.G; ++g) {
      const int64_t st = p.leaf_stride[i][g];
      if (st == 0) continue;
      if (!s.empty()) s += " + ";
      s += coord[g] + (st == 1 ? "" : " * " + std::to_string(st) + "u");
    }
    return s.empty() ? "0" : "(" + s + ")";
  }

  void gen_elementwise(const std::string& name) {
    prologue(name);
    const int G = p.G;
    os << "  const " << I << " NV = " << p.n / vec << "u;\n";
    os << "  for (" << I << " v = blockIdx.x * " << kThreads << "u + threadIdx.x; v < NV; v += gridDim.x * " << kThreads << "u) {\n";
    os << "    " << I << " e = v * " << vec << "u;\n";
    std::vector<std::string> coord(G);
    for (int g = G - 1; g >= 1; --g) {
      coord[g] = "c" + std::to_string(g);
      os << "    const " << I << " " << coord[g] << " = e % " << p.size[g] << "u; e /= " << p.size[g] << "u;\n";
    }
    coord[0] = "e";
    std::vector<std::string> loff(h.leaves.size());
    for (size_t i = 0; i < h.leaves.size(); ++i) loff[i] = leaf_offset((int)i, coord);
    for (int m = 0; m < (int)h.nodes.size(); ++m) emit_node(m, "", loff);
    emit_full_outputs("", "v * " + std::to_string(vec) + "u");
    os << "  }\n}\n";
  }

  // Marks in `need` the nodes an expression rooted at `m` recomputes inside
  // a walk along the row: those varying along it, up to (not into) values
  // that are constant per row (hoisted nodes and row reductions).
  void mark_row_nodes(int m, std::vector<char>& need) const {
    if (need[m] || !varies[m][p.G - 1]) return;
    const lmpb_fnode& nd = h.nodes[m];
    if (nd.kind == LMPB_FN_ROWRED) return;
    need[m] = 1;
    if (nd.kind == LMPB_FN_BINARY) {
      mark_row_nodes(nd.a, need);
      mark_row_nodes(nd.b, need);
    } else if (nd.kind == LMPB_FN_UNARY) {
      mark_row_nodes(nd.a, need);
    }
  }

  // Row reduce over group 1 of [P, Q]: one warp (short rows) or CTA per row.
  // In-kernel row reductions (LMPB_FN_ROWRED, e.g. the max and the sum of a
  // softmax) run as walks along the row before the final one, each followed
  // by the same warp/CTA tree as a reduce output and broadcast to the row's
  // threads, so a fused value equals the separately realized reduction bit
  // for bit.  Nodes constant along the row are computed once per row, as
  // soon as the row reductions they read are known.
  void gen_row_reduce(const std::string& name) {
    prologue(name);
    const int64_t P = p.size[0], Q = p.size[1];
    const bool W = p.warp_rows;
    const std::string tpr = W ? "32u" : std::to_string(kThreads) + "u";
    const int NN = (int)h.nodes.size();
    for (size_t j = 0; j < h.outs.size(); ++j)
      if (p.out_mode[j] >= LMPB_OUT_REDUCE_SUM)
        os << "  __shared__ " << tname(h.outs[j].dtype) << " sred" << j << "[" << kThreads / 32 << "];\n";
    std::vector<int> rr;  // row reductions in order
    std::vector<int> phase(NN, 0);
    for (int m = 0; m < NN; ++m) {
      const lmpb_fnode& nd = h.nodes[m];
      if (nd.kind == LMPB_FN_ROWRED) {
        rr.push_back(m);
        phase[m] = (int)rr.size();
        if (!W) {
          const std::string T = tname(nd.dtype);
          os << "  __shared__ " << T << " srr" << m << "[" << kThreads / 32 << "];\n  __shared__ " << T << " sbc" << m << ";\n";
        }
      } else if (nd.kind == LMPB_FN_BINARY) {
        phase[m] = std::max(phase[nd.a], phase[nd.b]);
      } else if (nd.kind == LMPB_FN_UNARY) {
        phase[m] = phase[nd.a];
      }
    }
    os << "  const unsigned lane = threadIdx.x & 31u, wid = threadIdx.x >> 5;\n";
    if (W)
      os << "  for (" << I << " row = blockIdx.x * " << kThreads / 32 << "u + wid; row < " << P << "u; row += gridDim.x * " << kThreads / 32 << "u) {\n"
         << "    const unsigned t = lane;\n";
    else
      os << "  for (" << I << " row = blockIdx.x; row < " << P << "u; row += gridDim.x) {\n"
         << "    const unsigned t = threadIdx.x;\n";
    std::vector<std::string> coord = {"row", "q"};
    std::vector<std::string> loff(h.leaves.size());
    for (size_t i = 0; i < h.leaves.size(); ++i) loff[i] = leaf_offset((int)i, coord);
    std::vector<char> done(NN, 0);
    auto hoist = [&](int upto) {  // per-row nodes whose row reductions are known
      for (int m = 0; m < NN; ++m)
        if (!done[m] && !varies[m][1] && h.nodes[m].kind != LMPB_FN_ROWRED && phase[m] <= upto) {
          emit_node(m, "", loff);
          done[m] = 1;
        }
    };
    auto walk_open = [&]() {
      if (p.row_unroll > 1) os << "    #pragma unroll " << p.row_unroll << "\n";
      os << "    for (" << I << " q = t * " << vec << "u; q < " << Q << "u; q += " << tpr << " * " << vec << "u) {\n";
    };
    for (size_t k = 0; k < rr.size(); ++k) {
      hoist((int)k);
      const int r = rr[k];
      const lmpb_fnode& nd = h.nodes[r];
      const std::string T = tname(nd.dtype), a = "racc" + std::to_string(r);
      const bool mx = nd.sub == LMPB_MAX;
      const std::string ident = mx ? "lmpb_dev::lowest<" + T + ">()" : T + "(0)";
      if (!varies[nd.a][1]) {  // a row reduction of a value constant along the row
        os << "    " << T << " " << a << " = " << ident << ";\n";
      } else {
        os << "    " << T << " " << a << " = " << ident << ";\n";
        std::vector<char> need(NN, 0);
        mark_row_nodes(nd.a, need);
        walk_open();
        for (int m = 0; m < NN; ++m)
          if (need[m]) emit_node(m, "  ", loff);
        const std::string x = "static_cast<" + T + ">(" + ref(nd.a, vec > 1) + ")";
        const std::string upd = mx ? a + " = (" + a + " < " + x + ") ? " + x + " : " + a + ";"
                                   : a + " = lmpb_dev::r_add<" + T + ">(" + a + ", " + x + ");";
        if (vec > 1)
          os << "      #pragma unroll\n      for (int j = 0; j < " << vec << "; ++j) " << upd << "\n";
        else
          os << "      " << upd << "\n";
        os << "    }\n";
      }
      if (!varies[nd.a][1]) {
        // sum over Q copies, or the value itself for max: as the reduce
        // output of a constant would compute it (a sequential walk per thread
        // and the tree), recomputed here the same way
        walk_open();
        const std::string x = "static_cast<" + T + ">(" + ref(nd.a, false) + ")";
        const std::string upd = mx ? a + " = (" + a + " < " + x + ") ? " + x + " : " + a + ";"
                                   : a + " = lmpb_dev::r_add<" + T + ">(" + a + ", " + x + ");";
        if (vec > 1) os << "      #pragma unroll\n      for (int j = 0; j < " << vec << "; ++j) " << upd << "\n";
        else os << "      " << upd << "\n";
        os << "    }\n";
      }
      const std::string red = mx ? "warp_max" : "warp_sum";
      os << "    " << a << " = " << red << "(" << a << ");\n";
      if (W) {
        os << "    const " << T << " v" << r << " = __shfl_sync(0xffffffffu, " << a << ", 0);\n";
      } else {
        os << "    if (lane == 0) srr" << r << "[wid] = " << a << ";\n    __syncthreads();\n";
        os << "    if (wid == 0) { " << a << " = lane < " << kThreads / 32 << "u ? srr" << r << "[lane] : " << ident << "; "
           << a << " = " << red << "(" << a << "); if (lane == 0) sbc" << r << " = " << a << "; }\n    __syncthreads();\n";
        os << "    const " << T << " v" << r << " = sbc" << r << ";\n    __syncthreads();\n";
      }
      done[r] = 1;
    }
    hoist((int)rr.size());
    for (size_t j = 0; j < h.outs.size(); ++j)
      if (p.out_mode[j] >= LMPB_OUT_REDUCE_SUM)
        os << "    " << tname(h.outs[j].dtype) << " acc" << j << " = 0;\n";
    walk_open();
    for (int m = 0; m < NN; ++m)
      if (!done[m]) emit_node(m, "  ", loff);
    emit_full_outputs("  ", "row * " + std::to_string(Q) + "u + q");
    for (size_t j = 0; j < h.outs.size(); ++j) {
      if (p.out_mode[j] < LMPB_OUT_REDUCE_SUM) continue;
      const std::string OT = tname(h.outs[j].dtype);
      const int m = h.outs[j].node;
      if (vec > 1)
        os << "      #pragma unroll\n      for (int j = 0; j < " << vec << "; ++j) acc" << j << " = lmpb_dev::r_add<" << OT
           << ">(acc" << j << ", static_cast<" << OT << ">(" << ref(m, true) << "));\n";
      else
        os << "      acc" << j << " = lmpb_dev::r_add<" << OT << ">(acc" << j << ", static_cast<" << OT << ">(" << ref(m, false) << "));\n";
    }
    os << "    }\n";
    // tree reduction and write
    for (size_t j = 0; j < h.outs.size(); ++j) {
      if (p.out_mode[j] < LMPB_OUT_REDUCE_SUM) continue;
      const std::string OT = tname(h.outs[j].dtype);
      const std::string a = "acc" + std::to_string(j);
      const std::string O = "O" + std::to_string(j);
      // output offset along P (group 0)
      const std::string oo = p.out_stride[j][0] == 0 ? "0" : "row * " + std::to_string(p.out_stride[j][0]) + "u";
      const int ad = h.outs[j].addend;
      const std::string val = ad >= 0 ? "lmpb_dev::r_add<" + OT + ">(static_cast<" + OT + ">(v" + std::to_string(ad) + "), " + a + ")" : a;
      std::string wr = p.out_mode[j] == LMPB_OUT_REDUCE_SUM_ACCUM
                           ? O + "[" + oo + "] = lmpb_dev::r_add<" + OT + ">(" + O + "[" + oo + "], " + val + ");"
                           : O + "[" + oo + "] = " + val + ";";
      os << "    " << a << " = warp_sum(" << a << ");\n";
      if (W) {
        os << "    if (lane == 0) " << wr << "\n";
      } else {
        os << "    if (lane == 0) sred" << j << "[wid] = " << a << ";\n    __syncthreads();\n";
        os << "    if (wid == 0) { " << a << " = lane < " << kThreads / 32 << "u ? sred" << j << "[lane] : " << OT << "(0); "
           << a << " = warp_sum(" << a << "); if (lane == 0) " << wr << " }\n    __syncthreads();\n";
      }
    }
    os << "  }\n}\n";
  }

  // Column reduce over group 0 of [P, Q], rows split into S chunks.
  void gen_col_reduce(const std::string& name) {
    prologue(name);
    const int64_t P = p.size[0], Q = p.size[1];
    const int64_t rpc = (P + p.S - 1) / p.S;
    os << "  const " << I << " q = (blockIdx.x * " << kThreads << "u + threadIdx.x) * " << vec << "u;\n";
    os << "  if (q >= " << Q << "u) return;\n";
    os << "  const " << I << " r0 = blockIdx.y * " << rpc << "u;\n";
    os << "  const " << I << " r1 = r0 + " << rpc << "u < " << P << "u ? r0 + " << rpc << "u : " << P << "u;\n";
    os << "  const " << I << " row = 0;\n";  // hoisted nodes do not depend on row
    std::vector<std::string> coord = {"row", "q"};
    std::vector<std::string> loff(h.leaves.size());
    for (size_t i = 0; i < h.leaves.size(); ++i) loff[i] = leaf_offset((int)i, coord);
    std::vector<char> done(h.nodes.size(), 0);
    for (int m = 0; m < (int)h.nodes.size(); ++m)
      if (!varies[m][0]) { emit_node(m, "", loff); done[m] = 1; }
    for (size_t j = 0; j < h.outs.size(); ++j)
      if (p.out_mode[j] >= LMPB_OUT_REDUCE_SUM) {
        const std::string OT = tname(h.outs[j].dtype);
        os << "  " << OT << " acc" << j << "[" << vec << "];\n  #pragma unroll\n  for (int j = 0; j < " << vec << "; ++j) acc" << j << "[j] = 0;\n";
      }
    os << "  for (" << I << " r = r0; r < r1; ++r) {\n";
    os << "    const " << I << " row = r;\n";
    for (int m = 0; m < (int)h.nodes.size(); ++m)
      if (!done[m]) emit_node(m, "", loff);
    emit_full_outputs("", "row * " + std::to_string(Q) + "u + q");
    for (size_t j = 0; j < h.outs.size(); ++j) {
      if (p.out_mode[j] < LMPB_OUT_REDUCE_SUM) continue;
      const std::string OT = tname(h.outs[j].dtype);
      const int m = h.outs[j].node;
      os << "    #pragma unroll\n    for (int j = 0; j < " << vec << "; ++j) acc" << j << "[j] = lmpb_dev::r_add<" << OT
         << ">(acc" << j << "[j], static_cast<" << OT << ">(" << ref(m, true) << "));\n";
    }
    os << "  }\n";
    for (size_t j = 0; j < h.outs.size(); ++j) {
      if (p.out_mode[j] < LMPB_OUT_REDUCE_SUM) continue;
      const std::string OT = tname(h.outs[j].dtype);
      const std::string O = "O" + std::to_string(j);
      const int ad = h.outs[j].addend;
      const std::string acc = "acc" + std::to_string(j) + "[j]";
      const std::string val = ad >= 0 ? "lmpb_dev::r_add<" + OT + ">(static_cast<" + OT + ">(" + ref(ad, true) + "), " + acc + ")" : acc;
      if (p.S > 1) {
        // chunk 0 carries the addend; the combine kernel sums chunks in order
        os << "  { " << OT << "* W = reinterpret_cast<" << OT << "*>(static_cast<char*>(prm.ws) + " << h.ws_offset[j] << "ull);\n"
           << "    #pragma unroll\n    for (int j = 0; j < " << vec << "; ++j) W[blockIdx.y * " << Q << "ull + q + j] = "
           << (ad >= 0 ? "blockIdx.y == 0 ? " + val + " : " + acc : acc) << "; }\n";
      } else {
        const std::string oo = "q + j";
        os << "  #pragma unroll\n  for (int j = 0; j < " << vec << "; ++j) ";
        if (p.out_mode[j] == LMPB_OUT_REDUCE_SUM_ACCUM)
          os << O << "[" << oo << "] = lmpb_dev::r_add<" << OT << ">(" << O << "[" << oo << "], " << val << ");\n";
        else
          os << O << "[" << oo << "] = " << val << ";\n";
      }
    }
    os << "}\n";
  }

  // Split-row partials -> outputs.  A CTA owns 32 adjacent columns; its 8 warps
  // each sum a contiguous run of chunks (8 loads in flight), and warp 0 folds
  // the 8 runs in order: deterministic, and not latency-bound on long S.
  void gen_combine(const std::string& name) {
    const int64_t Q = p.size[1];
    const int64_t per = (p.S + 7) / 8;
    os << "extern \"C\" __global__ void __launch_bounds__(" << kThreads << ") " << name << "(const Params prm) {\n";
    os << "  const unsigned lane = threadIdx.x & 31u, w = threadIdx.x >> 5;\n";
    os << "  const unsigned long long q = blockIdx.x * 32ull + lane;\n";
    os << "  const int s0 = (int)w * " << per << ", s1 = s0 + " << per << " < " << p.S << " ? s0 + " << per << " : " << p.S << ";\n";
    for (size_t j = 0; j < h.outs.size(); ++j) {
      if (p.out_mode[j] < LMPB_OUT_REDUCE_SUM) continue;
      const std::string OT = tname(h.outs[j].dtype);
      const std::string J = std::to_string(j);
      os << "  { __shared__ " << OT << " run" << J << "[8][32];\n";
      os << "    const " << OT << "* W = reinterpret_cast<const " << OT << "*>(static_cast<const char*>(prm.ws) + " << h.ws_offset[j] << "ull);\n";
      os << "    " << OT << " a = 0;\n";
      os << "    if (q < " << Q << "ull) {\n      int s = s0;\n";
      os << "      for (; s + 7 < s1; s += 8) { " << OT << " v[8];\n";
      os << "        #pragma unroll\n        for (int u = 0; u < 8; ++u) v[u] = W[(unsigned long long)(s + u) * " << Q << "ull + q];\n";
      os << "        #pragma unroll\n        for (int u = 0; u < 8; ++u) a = lmpb_dev::r_add<" << OT << ">(a, v[u]); }\n";
      os << "      for (; s < s1; ++s) a = lmpb_dev::r_add<" << OT << ">(a, W[(unsigned long long)s * " << Q << "ull + q]);\n    }\n";
      os << "    run" << J << "[w][lane] = a;\n    __syncthreads();\n";
      os << "    if (w == 0 && q < " << Q << "ull) { " << OT << " r = run" << J << "[0][lane];\n";
      os << "      #pragma unroll\n      for (int k = 1; k < 8; ++k) r = lmpb_dev::r_add<" << OT << ">(r, run" << J << "[k][lane]);\n";
      os << "      " << OT << "* O = static_cast<" << OT << "*>(prm.out[" << J << "]);\n";
      if (p.out_mode[j] == LMPB_OUT_REDUCE_SUM_ACCUM)
        os << "      O[q] = lmpb_dev::r_add<" << OT << ">(O[q], r);\n";
      else
        os << "      O[q] = r;\n";
      os << "    }\n    __syncthreads();\n  }\n";
    }
    os << "}\n";
  }
};

std::string generate(lmpb_fused_s& h) {
  std::ostringstream src;
  src << "// generated by lmpb fused compiler\n" << kOpsDeviceSource << "\n";
  src << "template <typename T, int V> struct alignas(sizeof(T) * V >= 16 ? 16 : sizeof(T) * V) Pack { T v[V]; };\n";
  // evict-first (streaming) 16-byte accesses, for data touched once per pass
  src << "template <typename T, int V> __device__ __forceinline__ void st_cs(T* p, const Pack<T, V>& v) {\n"
         "  const uint4* s = reinterpret_cast<const uint4*>(&v); uint4* d = reinterpret_cast<uint4*>(p);\n"
         "  #pragma unroll\n  for (int i = 0; i < (int)(sizeof(Pack<T, V>) / 16); ++i) __stcs(d + i, s[i]);\n}\n"
         "template <typename T, int V> __device__ __forceinline__ Pack<T, V> ld_cs(const T* p) {\n"
         "  Pack<T, V> v; uint4* d = reinterpret_cast<uint4*>(&v); const uint4* s = reinterpret_cast<const uint4*>(p);\n"
         "  #pragma unroll\n  for (int i = 0; i < (int)(sizeof(Pack<T, V>) / 16); ++i) d[i] = __ldcs(s + i);\n  return v;\n}\n";
  src << "template <typename T> __device__ __forceinline__ T warp_sum(T v) {\n"
         "  #pragma unroll\n  for (int d = 16; d > 0; d >>= 1) v = lmpb_dev::r_add<T>(v, static_cast<T>(__shfl_down_sync(0xffffffffu, v, d)));\n"
         "  return v;\n}\n";
  src << "template <typename T> __device__ __forceinline__ T warp_max(T v) {\n"
         "  #pragma unroll\n  for (int d = 16; d > 0; d >>= 1) { T o = static_cast<T>(__shfl_down_sync(0xffffffffu, v, d)); v = (v < o) ? o : v; }\n"
         "  return v;\n}\n";
  src << "template <> __device__ __forceinline__ bool warp_sum<bool>(bool v) { return __any_sync(0xffffffffu, v); }\n";
  src << "template <> __device__ __forceinline__ short warp_sum<short>(short v) { int x = v;\n"
         "  for (int d = 16; d > 0; d >>= 1) x = (short)(x + __shfl_down_sync(0xffffffffu, x, d)); return (short)x; }\n";
  src << "struct Params { const void* leaf[" << std::max<size_t>(1, h.leaves.size()) << "]; void* out["
      << std::max<size_t>(1, h.outs.size()) << "]; void* ws; };\n";
  const Plan& p = h.plan;
  for (int variant = 0; variant < 2; ++variant) {
    const int vec = variant == 0 ? p.vec : 1;
    Gen g(h, vec);
    const std::string name = variant == 0 ? "lmpb_fused_v" : "lmpb_fused_s";
    if (p.pattern == kElementwise) g.gen_elementwise(name);
    else if (p.pattern == kRowReduce) g.gen_row_reduce(name);
    else g.gen_col_reduce(name);
    src << g.os.str();
  }
  if (p.pattern == kColReduce && p.S > 1) {
    Gen g(h, 1);
    g.gen_combine("lmpb_fused_c");
    src << g.os.str();
  }
  return src.str();
}

// ------------------------------------------------------------ compile cache

struct Cubin {
  std::vector<char> bytes;
};

std::mutex g_cache_mu;
std::map<std::string, std::shared_ptr<Cubin>>& mem_cache() {
  static auto* m = new std::map<std::string, std::shared_ptr<Cubin>>();
  return *m;
}

std::string cache_dir() {
  const char* e = getenv("LMPB_KERNEL_CACHE");
  std::string d;
  if (e && *e) d = e;
  else {
    const char* home = getenv("HOME");
    d = std::string(home && *home ? home : "/tmp") + "/.cache/lmpb_b200";
  }
  return d;
}

void mkdirs(const std::string& d) {
  std::string cur;
  std::stringstream ss(d);
  std::string part;
  if (!d.empty() && d[0] == '/') cur = "/";
  while (std::getline(ss, part, '/')) {
    if (part.empty()) continue;
    cur += part + "/";
    mkdir(cur.c_str(), 0755);
  }
}

bool read_file(const std::string& path, std::string& out) {
  std::ifstream f(path, std::ios::binary);
  if (!f) return false;
  std::ostringstream ss;
  ss << f.rdbuf();
  out = ss.str();
  return true;
}

void write_atomic(const std::string& path, const std::string& data) {
  std::string tmp = path + ".tmp." + std::to_string(getpid());
  {
    std::ofstream f(tmp, std::ios::binary);
    if (!f) return;
    f.write(data.data(), (std::streamsize)data.size());
  }
  rename(tmp.c_str(), path.c_str());
}

lmpb_status compile(const std::string& src, std::shared_ptr<Cubin>& out) {
  {
    std::lock_guard<std::mutex> lk(g_cache_mu);
    auto it = mem_cache().find(src);
    if (it != mem_cache().end()) {
      out = it->second;
      return LMPB_OK;
    }
  }
  int major = 0, minor = 0;
  nvrtcVersion(&major, &minor);
  const std::string key_src = src + "\n// nvrtc " + std::to_string(major) + "." + std::to_string(minor) + " sm_100a";
  char hex[32];
  snprintf(hex, sizeof hex, "%016llx", (unsigned long long)fnv1a(key_src));
  const std::string dir = cache_dir();
  const std::string base = dir + "/" + hex;
  std::string disk_src, disk_bin;
  if (read_file(base + ".cu", disk_src) && disk_src == key_src && read_file(base + ".cubin", disk_bin) &&
      !disk_bin.empty()) {
    auto c = std::make_shared<Cubin>();
    c->bytes.assign(disk_bin.begin(), disk_bin.end());
    std::lock_guard<std::mutex> lk(g_cache_mu);
    mem_cache()[src] = c;
    out = c;
    return LMPB_OK;
  }
  if (getenv("LMPB_FUSED_LOG")) fprintf(stderr, "[lmpb fused] NVRTC compile %s (%zu bytes of source)\n", hex, src.size());
  nvrtcProgram prog;
  if (nvrtcCreateProgram(&prog, src.c_str(), "lmpb_fused.cu", 0, nullptr, nullptr) != NVRTC_SUCCESS)
    return set_error(LMPB_ERR_COMPILE, "nvrtcCreateProgram failed");
  const char* opts[] = {"--gpu-architecture=sm_100a", "-std=c++17", "--fmad=false", "-default-device",
                        "-lineinfo"};
  nvrtcResult r = nvrtcCompileProgram(prog, 5, opts);
  if (r != NVRTC_SUCCESS) {
    size_t n = 0;
    nvrtcGetProgramLogSize(prog, &n);
    std::string log(n, '\0');
    nvrtcGetProgramLog(prog, &log[0]);
    nvrtcDestroyProgram(&prog);
    return set_error(LMPB_ERR_COMPILE, "NVRTC compile failed:\n" + log + "\n--- source ---\n" + src);
  }
  size_t n = 0;
  nvrtcGetCUBINSize(prog, &n);
  auto c = std::make_shared<Cubin>();
  c->bytes.resize(n);
  nvrtcGetCUBIN(prog, c->bytes.data());
  nvrtcDestroyProgram(&prog);
  mkdirs(dir);
  write_atomic(base + ".cubin", std::string(c->bytes.begin(), c->bytes.end()));
  write_atomic(base + ".cu", key_src);
  std::lock_guard<std::mutex> lk(g_cache_mu);
  mem_cache()[src] = c;
  out = c;
  return LMPB_OK;
}

// Driver entry points, resolved through the runtime so that the library does
// not link libcuda directly (it loads on machines without a driver, e.g. a
// build host; the calls below only run once a GPU is present).
struct Driver {
  CUresult (*ctxGetCurrent)(CUcontext*) = nullptr;
  CUresult (*moduleLoadData)(CUmodule*, const void*) = nullptr;
  CUresult (*moduleGetFunction)(CUfunction*, CUmodule, const char*) = nullptr;
  CUresult (*launchKernel)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned,
                           unsigned, CUstream, void**, void**) = nullptr;
  CUresult (*getErrorString)(CUresult, const char**) = nullptr;
  bool ok = false;
};

template <typename F>
bool resolve(const char* name, F& fn) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || !p)
    return false;
  fn = reinterpret_cast<F>(p);
  return true;
}

const Driver& drv() {
  static Driver d = [] {
    Driver x;
    cudaFree(nullptr);
    x.ok = resolve("cuCtxGetCurrent", x.ctxGetCurrent) && resolve("cuModuleLoadData", x.moduleLoadData) &&
           resolve("cuModuleGetFunction", x.moduleGetFunction) && resolve("cuLaunchKernel", x.launchKernel) &&
           resolve("cuGetErrorString", x.getErrorString);
    return x;
  }();
  return d;
}

lmpb_status cu_err(CUresult r, const char* what) {
  const char* s = nullptr;
  if (drv().getErrorString) drv().getErrorString(r, &s);
  return set_error(LMPB_ERR_CUDA, std::string(what) + ": " + (s ? s : "unknown CUDA driver error"));
}

lmpb_status get_functions(lmpb_fused_s& h, std::array<CUfunction, 3>& fns) {
  if (!drv().ok) return set_error(LMPB_ERR_CUDA, "fused: CUDA driver entry points unavailable");
  CUcontext ctx = nullptr;
  CUresult r = drv().ctxGetCurrent(&ctx);
  if (r == CUDA_SUCCESS && ctx == nullptr) {
    cudaFree(nullptr);  // first runtime call on this thread: make the primary context current
    r = drv().ctxGetCurrent(&ctx);
  }
  if (r != CUDA_SUCCESS || ctx == nullptr) return set_error(LMPB_ERR_CUDA, "fused: no current CUDA context");
  std::lock_guard<std::mutex> lk(h.mu);
  auto it = h.fn.find(ctx);
  if (it != h.fn.end()) {
    fns = it->second;
    return LMPB_OK;
  }
  std::shared_ptr<Cubin> cub;
  lmpb_status st = compile(h.source, cub);
  if (st != LMPB_OK) return st;
  CUmodule mod;
  r = drv().moduleLoadData(&mod, cub->bytes.data());
  if (r != CUDA_SUCCESS) return cu_err(r, "cuModuleLoadData");
  std::array<CUfunction, 3> f{};
  if ((r = drv().moduleGetFunction(&f[0], mod, "lmpb_fused_v")) != CUDA_SUCCESS) return cu_err(r, "cuModuleGetFunction");
  if ((r = drv().moduleGetFunction(&f[1], mod, "lmpb_fused_s")) != CUDA_SUCCESS) return cu_err(r, "cuModuleGetFunction");
  if (h.plan.pattern == kColReduce && h.plan.S > 1)
    if ((r = drv().moduleGetFunction(&f[2], mod, "lmpb_fused_c")) != CUDA_SUCCESS) return cu_err(r, "cuModuleGetFunction");
  h.fn[ctx] = f;
  fns = f;
  return LMPB_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" lmpb_status lmpb_fused_build(const lmpb_fnode* nodes, int n_nodes, const lmpb_fleaf* leaves,
                                        int n_leaves, const lmpb_fout* outs, int n_outs,
                                        const int64_t* iter_shape, int iter_ndim, lmpb_fused* handle) {
  if (!handle) return set_error(LMPB_ERR_INVALID, "fused: null handle");
  *handle = nullptr;
  if (n_nodes <= 0 || n_outs <= 0 || n_leaves < 0 || !nodes || !outs || (n_leaves && !leaves))
    return set_error(LMPB_ERR_INVALID, "fused: empty program");
  if (iter_ndim < 0 || iter_ndim > LMPB_MAX_DIMS || (iter_ndim && !iter_shape))
    return set_error(LMPB_ERR_INVALID, "fused: bad iteration shape");
  for (int i = 0; i < iter_ndim; ++i)
    if (iter_shape[i] < 0) return set_error(LMPB_ERR_INVALID, "fused: negative extent");
  for (int m = 0; m < n_nodes; ++m) {
    const lmpb_fnode& nd = nodes[m];
    if (!lmpb::valid_dtype(nd.dtype)) return set_error(LMPB_ERR_INVALID, "fused: node dtype");
    switch (nd.kind) {
      case LMPB_FN_LEAF:
        if (nd.a < 0 || nd.a >= n_leaves) return set_error(LMPB_ERR_INVALID, "fused: leaf slot out of range");
        break;
      case LMPB_FN_CONST: break;
      case LMPB_FN_BINARY:
        if (nd.sub < LMPB_ADD || nd.sub > LMPB_CLAMP_BACKWARD || nd.a < 0 || nd.a >= m || nd.b < 0 || nd.b >= m)
          return set_error(LMPB_ERR_INVALID, "fused: bad binary node");
        break;
      case LMPB_FN_UNARY:
        if (nd.sub < LMPB_NEG || nd.sub > LMPB_CLAMP || nd.a < 0 || nd.a >= m)
          return set_error(LMPB_ERR_INVALID, "fused: bad unary node");
        break;
      case LMPB_FN_ROWRED:
        if ((nd.sub != LMPB_SUM && nd.sub != LMPB_MAX) || nd.a < 0 || nd.a >= m)
          return set_error(LMPB_ERR_INVALID, "fused: bad row-reduction node");
        break;
      default: return set_error(LMPB_ERR_INVALID, "fused: unknown node kind");
    }
  }
  for (int i = 0; i < n_leaves; ++i)
    if (!lmpb::valid_dtype(leaves[i].dtype) || leaves[i].ndim < 0 || leaves[i].ndim > LMPB_MAX_DIMS)
      return set_error(LMPB_ERR_INVALID, "fused: bad leaf");
  for (int j = 0; j < n_outs; ++j)
    if (outs[j].node < 0 || outs[j].node >= n_nodes || !lmpb::valid_dtype(outs[j].dtype) ||
        outs[j].mode < LMPB_OUT_STORE || outs[j].mode > LMPB_OUT_REDUCE_SUM_ACCUM || outs[j].ndim < 0 ||
        outs[j].ndim > LMPB_MAX_DIMS)
      return set_error(LMPB_ERR_INVALID, "fused: bad output");
  auto h = std::make_unique<lmpb_fused_s>();
  h->nodes.assign(nodes, nodes + n_nodes);
  h->leaves.assign(leaves, leaves + n_leaves);
  h->outs.assign(outs, outs + n_outs);
  lmpb_status st = make_plan(*h, iter_shape, iter_ndim);
  if (st != LMPB_OK) return st;
  {
    Gen g(*h, 1);
    for (int j = 0; j < n_outs; ++j) {
      const int ad = outs[j].addend;
      if (ad < 0) continue;
      const int mode = h->plan.out_mode[j];
      if (ad >= n_nodes || mode < LMPB_OUT_REDUCE_SUM)
        return set_error(LMPB_ERR_INVALID, "fused: an addend needs a reduce output");
      for (int gi = 0; gi < h->plan.G; ++gi)
        if (h->plan.out_stride[j][gi] == 0 && h->plan.size[gi] > 1 && g.varies[ad][gi])
          return set_error(LMPB_ERR_INVALID, "fused: the addend varies along a reduced axis");
    }
  }
  h->ws_offset.assign(n_outs, 0);
  if (h->plan.pattern == kColReduce && h->plan.S > 1) {
    size_t off = 0;
    for (int j = 0; j < n_outs; ++j) {
      if (h->plan.out_mode[j] < LMPB_OUT_REDUCE_SUM) continue;
      h->ws_offset[j] = off;
      off += ((size_t)h->plan.S * h->plan.size[1] * lmpb::dtype_size(outs[j].dtype) + 255) / 256 * 256;
    }
    h->ws_bytes = off;
  }
  h->source = generate(*h);
  *handle = h.release();
  return LMPB_OK;
}

extern "C" lmpb_status lmpb_fused_launch(lmpb_fused h, const void* const* leaf_ptrs, void* const* out_ptrs,
                                         void* stream) {
  if (!h) return set_error(LMPB_ERR_INVALID, "fused: null handle");
  const Plan& p = h->plan;
  if (p.n == 0) return LMPB_OK;
  std::array<CUfunction, 3> fns;
  lmpb_status st = get_functions(*h, fns);
  if (st != LMPB_OK) return st;
  const int NL = (int)h->leaves.size(), NO = (int)h->outs.size();
  // parameter block: leaf pointers, output pointers, workspace pointer
  std::vector<void*> prm(std::max(1, NL) + std::max(1, NO) + 1, nullptr);
  bool al = true;
  for (int i = 0; i < NL; ++i) {
    if (!leaf_ptrs || !leaf_ptrs[i]) return set_error(LMPB_ERR_INVALID, "fused: null leaf pointer");
    prm[i] = const_cast<void*>(leaf_ptrs[i]);
    al = al && aligned16(leaf_ptrs[i]);
  }
  const int ob = std::max(1, NL);
  for (int j = 0; j < NO; ++j) {
    if (!out_ptrs || !out_ptrs[j]) return set_error(LMPB_ERR_INVALID, "fused: null output pointer");
    prm[ob + j] = out_ptrs[j];
    al = al && aligned16(out_ptrs[j]);
  }
  cudaStream_t cst = reinterpret_cast<cudaStream_t>(stream);
  void* ws = nullptr;
  if (h->ws_bytes) {
    cudaError_t e = lmpb::stream_alloc(&ws, h->ws_bytes, cst);
    if (e != cudaSuccess) return set_error(LMPB_ERR_CUDA, std::string("fused workspace: ") + cudaGetErrorString(e));
  }
  prm[ob + std::max(1, NO)] = ws;
  void* args[] = {prm.data()};
  const bool use_vec = al && p.vec > 1;
  CUfunction f = use_vec ? fns[0] : fns[1];
  const int vec = use_vec ? p.vec : 1;
  const int64_t cap = (int64_t)lmpb::sm_count() * 8;
  unsigned gx = 1, gy = 1;
  if (p.pattern == kElementwise) {
    int64_t b = (p.n / vec + kThreads - 1) / kThreads;
    gx = (unsigned)std::max<int64_t>(1, std::min(b, cap));
  } else if (p.pattern == kRowReduce) {
    int64_t rows = p.size[0];
    int64_t b = p.warp_rows ? (rows + kThreads / 32 - 1) / (kThreads / 32) : rows;
    gx = (unsigned)std::max<int64_t>(1, std::min(b, cap));
  } else {
    gx = (unsigned)((p.size[1] / vec + kThreads - 1) / kThreads);
    gy = (unsigned)p.S;
  }
  // kernel parameters are passed as one struct: CU_LAUNCH_PARAM_BUFFER_POINTER
  size_t psize = prm.size() * sizeof(void*);
  void* config[] = {CU_LAUNCH_PARAM_BUFFER_POINTER, prm.data(), CU_LAUNCH_PARAM_BUFFER_SIZE, &psize,
                    CU_LAUNCH_PARAM_END};
  (void)args;
  CUresult r = drv().launchKernel(f, gx, gy, 1, kThreads, 1, 1, 0, reinterpret_cast<CUstream>(stream), nullptr, config);
  lmpb::count_launch();
  if (r != CUDA_SUCCESS) {
    if (ws) cudaFreeAsync(ws, cst);
    return cu_err(r, "cuLaunchKernel(fused)");
  }
  if (p.pattern == kColReduce && p.S > 1) {
    const unsigned g2 = (unsigned)((p.size[1] + 31) / 32);
    r = drv().launchKernel(fns[2], g2, 1, 1, kThreads, 1, 1, 0, reinterpret_cast<CUstream>(stream), nullptr, config);
    lmpb::count_launch();
    if (r != CUDA_SUCCESS) {
      cudaFreeAsync(ws, cst);
      return cu_err(r, "cuLaunchKernel(fused combine)");
    }
  }
  if (ws) {
    cudaError_t e = cudaFreeAsync(ws, cst);
    if (e != cudaSuccess) return set_error(LMPB_ERR_CUDA, std::string("fused workspace free: ") + cudaGetErrorString(e));
  }
  return LMPB_OK;
}

extern "C" lmpb_status lmpb_fused_release(lmpb_fused h) {
  delete h;  // modules stay loaded for the process lifetime (shared through the cubin cache)
  return LMPB_OK;
}

extern "C" const char* lmpb_fused_source(lmpb_fused h) { return h ? h->source.c_str() : ""; }
