// lower.cpp -- lowering of an extracted BAFE graph to launch steps and the
// CUDA source of their kernels.
//
// BAFE's emitter (codegen.c:172-534) gives every node its own buffer and a
// loop nest.  The extractor hands the backend unfused chains at practical
// sizes (matmul -> add -> relu; mul -> add -> relu), so this pass does the
// fusion a GPU needs:
//   * elementwise nodes (add/sub/mul/bias_add/relu/neg/sigmoid/tanh,
//     fused_bias_relu, reshape, layout_transform) are grouped into regions;
//     one region = one streaming kernel that reads each leaf once and writes
//     the region root once;
//   * a matmul whose only consumer chain is a region is fused into it: the
//     region becomes the GEMM's epilogue, evaluated on the accumulator
//     before the single store (relu(matmul(A,B)+C) is one kernel);
//   * transpose / broadcast_to / reductions / unknown ops get their own
//     steps.
// Per-element arithmetic is emitted with the C types and conversions the
// reference's C would apply (usual arithmetic conversions, assignment to
// the node's buffer type), so every elementwise result is bit-identical.
#include "internal.h"

#include <algorithm>
#include <cstdio>
#include <functional>
#include <map>
#include <set>
#include <sstream>

namespace bafe_cuda {

namespace {

enum Access { FULL = 0, ROW = 1 };

bool is_ew_op(Op op) {
    switch (op) {
        case Op::Add: case Op::Sub: case Op::Mul: case Op::BiasAdd: case Op::FusedBiasRelu:
        case Op::Relu: case Op::Neg: case Op::Sigmoid: case Op::Tanh:
        case Op::Reshape: case Op::LayoutTransform:
            return true;
        default:
            return false;
    }
}

bool is_gemm_op(Op op) {
    return op == Op::MatMul || op == Op::FusedMatmulRelu || op == Op::FusedMatmulBias ||
           op == Op::FusedMatmulBiasRelu;
}

// C's usual arithmetic conversions over the compute types the emitter uses.
int common_type(int a, int b) {
    if (a == BAFE_DTYPE_F64 || b == BAFE_DTYPE_F64) return BAFE_DTYPE_F64;
    if (a == BAFE_DTYPE_F32 || b == BAFE_DTYPE_F32) return BAFE_DTYPE_F32;
    if (a == BAFE_DTYPE_I64 || b == BAFE_DTYPE_I64) return BAFE_DTYPE_I64;
    return BAFE_DTYPE_I32;
}

const char* ctype(int compute) { return dtype_ctype(compute); }

bool is_float(int t) { return t == BAFE_DTYPE_F32 || t == BAFE_DTYPE_F64; }

std::string cast(int to, int from, const std::string& e) {
    if (to == from) return e;
    return std::string("((") + ctype(to) + ")(" + e + "))";
}

struct Lowerer {
    const Graph& G;
    const Options& opt;
    Plan& P;
    std::string& err;

    std::vector<char> reach;
    std::vector<std::vector<std::pair<int, int>>> cons;   // (consumer, child slot)
    std::vector<std::vector<int>> mode;                    // per node, per child slot
    std::vector<char> ew, mat;
    std::vector<int> fused_gemm;     // region root -> fused gemm node (-1)
    std::vector<int> fused_into;     // gemm node -> region root (-1)
    std::vector<BufRef> buf;
    std::vector<int> buf_dtype;      // stored dtype of the node's buffer
    std::vector<char> has_buf;
    std::ostringstream src;
    int kcount = 0;

    Lowerer(const Graph& g, const Options& o, Plan& p, std::string& e)
        : G(g), opt(o), P(p), err(e) {}

    const Node& N(int id) const { return G.nodes[id]; }
    int ct(int id) const { return compute_dtype(N(id).dtype); }

    // Access mode of child slot c of EW node n, following the emitter's
    // broadcast cases (codegen.c:302-326, 327-337, 518-528).  Returns -1 for
    // shapes the emitter would index out of range.
    int child_access(int n, int c) const {
        const Node& x = N(n);
        switch (x.op) {
            case Op::Add: case Op::Sub: case Op::Mul: {
                const Shape& a = N(x.ch[0]).shape;
                const Shape& b = N(x.ch[1]).shape;
                if (a.rank == 2 && b.rank == 1 && a.d[1] == b.d[0]) return c == 0 ? FULL : ROW;
                if (a.rank == 1 && b.rank == 2 && a.d[0] == b.d[1]) return c == 0 ? ROW : FULL;
                if (a.numel() == x.shape.numel() && b.numel() == x.shape.numel()) return FULL;
                return -1;
            }
            case Op::BiasAdd: case Op::FusedBiasRelu: {
                if (x.shape.rank != 2) return -1;
                if (c == 0) return N(x.ch[0]).shape.numel() == x.shape.numel() ? FULL : -1;
                return N(x.ch[1]).shape.numel() == x.shape.d[1] ? ROW : -1;
            }
            default:
                return N(x.ch[c]).shape.numel() == x.shape.numel() ? FULL : -1;
        }
    }

    int64_t ncols_of(int n) const {
        const Shape& s = N(n).shape;
        return s.rank ? std::max<int64_t>(s.d[s.rank - 1], 1) : 1;
    }

    // ----------------------------------------------------------- analysis --
    int analyse() {
        const int nn = (int)G.nodes.size();
        reach.assign(nn, 0);
        cons.assign(nn, {});
        mode.assign(nn, {});
        std::vector<int> stack{G.root};
        while (!stack.empty()) {
            int id = stack.back(); stack.pop_back();
            if (reach[id]) continue;
            reach[id] = 1;
            for (int c : N(id).ch) stack.push_back(c);
        }
        for (int id = 0; id < nn; ++id) {
            if (!reach[id]) continue;
            const Node& x = N(id);
            if (x.op == Op::Constant) {
                // The emitter never declares constant buffers, so any graph
                // that reads one fails to compile (codegen.c:175, 55-57).
                err = "constant nodes are not supported by the kernel emitter";
                return 2;
            }
            if (x.op == Op::Input && x.input_index < 0) {
                err = "input node '" + x.name + "' is not listed in the graph inputs";
                return 2;
            }
            for (size_t c = 0; c < x.ch.size(); ++c) cons[x.ch[c]].push_back({id, (int)c});
        }
        ew.assign(nn, 0);
        for (int id = 0; id < nn; ++id) {
            if (!reach[id]) continue;
            const Node& x = N(id);
            if (!is_ew_op(x.op)) continue;
            int arity = (x.op == Op::Add || x.op == Op::Sub || x.op == Op::Mul || x.op == Op::BiasAdd ||
                         x.op == Op::FusedBiasRelu) ? 2 : 1;
            if ((int)x.ch.size() != arity) { err = "node " + std::to_string(id) + " (" + x.opname + ") has the wrong arity"; return 2; }
            mode[id].resize(arity);
            for (int c = 0; c < arity; ++c) {
                int m = child_access(id, c);
                if (m < 0) {
                    err = "unsupported broadcast in node " + std::to_string(id) + " (" + x.opname + " of " +
                          N(x.ch[0]).shape.str() + (arity == 2 ? " and " + N(x.ch[1]).shape.str() : std::string()) +
                          "): the reference emitter reads out of range for these shapes";
                    return 2;
                }
                mode[id][c] = m;
            }
            ew[id] = 1;
        }
        // Materialisation: an EW node gets its own buffer when it is the
        // output, feeds a non-EW node, or is read as a row vector.
        mat.assign(nn, 0);
        for (int id = 0; id < nn; ++id) {
            if (!reach[id] || N(id).op == Op::Input) continue;
            if (!ew[id]) { mat[id] = 1; continue; }
            if (id == G.root) { mat[id] = 1; continue; }
            for (auto& cs : cons[id]) {
                if (!ew[cs.first] || mode[cs.first][cs.second] == ROW) { mat[id] = 1; break; }
            }
        }
        // GEMM epilogue fusion: a GEMM read by exactly one EW node (FULL),
        // whose chain of single-consumer non-materialised EW nodes ends at a
        // region root of the same element count.
        fused_gemm.assign(nn, -1);
        fused_into.assign(nn, -1);
        for (int id = 0; id < nn; ++id) {
            if (!reach[id] || !is_gemm_op(N(id).op) || id == G.root) continue;
            if (cons[id].size() != 1) continue;
            int c = cons[id][0].first;
            if (!ew[c] || mode[c][cons[id][0].second] != FULL) continue;
            while (!mat[c]) {
                if (cons[c].size() != 1) { c = -1; break; }
                c = cons[c][0].first;
            }
            if (c < 0 || !ew[c]) continue;
            if (N(c).shape.numel() != N(id).shape.numel()) continue;
            if (fused_gemm[c] >= 0) continue;
            fused_gemm[c] = id;
            fused_into[id] = c;
            mat[id] = 0;
        }
        // Operand limits of the generated kernels: a region reads at most
        // kRegionLeaves distinct operands, a GEMM epilogue at most
        // kEpilogueLeaves (fixed-size parameter blocks).  Wider expressions
        // are cut until every kernel fits: a GEMM whose epilogue would read
        // too many writes its product to a buffer of its own instead, and
        // an oversized region gets an internal node materialised: of the
        // nodes whose own region then fits, the one that leaves the fewest
        // operands to the rest (else the one that removes the most, and
        // the rest is cut again).  The emitter gives every node
        // a buffer anyway (codegen.c:188), so a cut adds a launch and
        // leaves every value as it was.
        for (bool changed = true; changed;) {
            changed = false;
            for (int id = 0; id < nn && !changed; ++id) {
                if (!reach[id] || !ew[id] || !mat[id]) continue;
                const Region R = collect_region(id);
                if (R.acc >= 0) {
                    const Op gop = N(R.acc).op;
                    const size_t bias = (gop == Op::FusedMatmulBias || gop == Op::FusedMatmulBiasRelu) ? 1 : 0;
                    if (R.leaves.size() + bias <= kEpilogueLeaves) continue;
                    fused_into[R.acc] = -1;
                    fused_gemm[id] = -1;
                    mat[R.acc] = 1;
                    changed = true;
                    continue;
                }
                if (R.leaves.size() <= kRegionLeaves) continue;
                int best = -1;
                bool best_fits = false;
                size_t best_n = R.leaves.size();
                for (int x : R.order) {
                    if (x == id) continue;
                    mat[x] = 1;
                    const size_t n = collect_region(id).leaves.size();
                    const bool fits = collect_region(x).leaves.size() <= kRegionLeaves;
                    mat[x] = 0;
                    if (n >= R.leaves.size()) continue;            // removes nothing
                    if ((fits && !best_fits) || (fits == best_fits && n < best_n)) {
                        best = x;
                        best_fits = fits;
                        best_n = n;
                    }
                }
                if (best >= 0) {
                    mat[best] = 1;
                } else {
                    for (int x : R.order) if (x != id) mat[x] = 1;   // no single cut helps: one kernel per node
                }
                changed = true;
            }
        }
        return 0;
    }
    static constexpr size_t kRegionLeaves = 16, kEpilogueLeaves = 8;

    // ------------------------------------------------------------ buffers --
    void assign_buffers() {
        const int nn = (int)G.nodes.size();
        buf.assign(nn, BufRef());
        buf_dtype.assign(nn, BAFE_DTYPE_F32);
        has_buf.assign(nn, 0);
        for (int id = 0; id < nn; ++id) {
            if (!reach[id]) continue;
            const Node& x = N(id);
            if (x.op == Op::Input) {
                buf[id] = {BufRef::In, x.input_index};
                buf_dtype[id] = x.dtype;
                has_buf[id] = 1;
            } else if (mat[id] && id != G.root) {
                buf[id] = {BufRef::Tmp, (int)P.tmp_bytes.size()};
                buf_dtype[id] = ct(id);
                P.tmp_bytes.push_back(x.shape.numel() * dtype_size(ct(id)));
                has_buf[id] = 1;
            }
        }
        buf[G.root] = {BufRef::Out, 0};
        buf_dtype[G.root] = N(G.root).dtype;
        has_buf[G.root] = 1;
        P.out_dtype = N(G.root).dtype;
        P.out_bytes = N(G.root).shape.numel() * dtype_size(N(G.root).dtype);
    }

    BufRef new_tmp(int64_t bytes) {
        BufRef r{BufRef::Tmp, (int)P.tmp_bytes.size()};
        P.tmp_bytes.push_back(bytes);
        return r;
    }

    static std::string bufname(const BufRef& b) {
        switch (b.kind) {
            case BufRef::In: return "in" + std::to_string(b.idx);
            case BufRef::Tmp: return "tmp" + std::to_string(b.idx);
            default: return "out";
        }
    }

    // Value expression of a leaf read: stored type -> compute type.
    static std::string load_convert(int stored_dtype, const std::string& e) {
        if (stored_dtype == BAFE_DTYPE_F16) return "bafe::f16_to_f32(" + e + ")";
        if (stored_dtype == BAFE_DTYPE_BF16) return "bafe::bf16_to_f32(" + e + ")";
        return e;
    }
    // Store expression: compute value -> stored type of the destination.
    static std::string store_convert(int stored_dtype, int compute, const std::string& e) {
        if (stored_dtype == BAFE_DTYPE_F16) return "bafe::f32_to_f16(" + cast(BAFE_DTYPE_F32, compute, e) + ")";
        if (stored_dtype == BAFE_DTYPE_BF16) return "bafe::f32_to_bf16(" + cast(BAFE_DTYPE_F32, compute, e) + ")";
        return cast(stored_dtype, compute, e);
    }

    // ------------------------------------------------------------ regions --
    struct Leaf { int node; int access; };
    struct Region {
        int root = -1;
        int acc = -1;                  // fused GEMM node (value = accumulator)
        std::vector<int> order;        // internal EW nodes, children first
        std::vector<Leaf> leaves;      // distinct (node, access) leaves
    };

    Region collect_region(int root) {
        Region R;
        R.root = root;
        R.acc = fused_gemm[root];
        std::set<int> seen;
        std::function<void(int)> visit = [&](int id) {
            if (seen.count(id)) return;
            seen.insert(id);
            const Node& x = N(id);
            for (size_t c = 0; c < x.ch.size(); ++c) {
                int ch = x.ch[c];
                int m = mode[id][c];
                bool internal = ew[ch] && !mat[ch] && m == FULL && ch != R.acc;
                if (internal) {
                    visit(ch);
                } else if (ch != R.acc) {
                    bool dup = false;
                    for (auto& l : R.leaves) if (l.node == ch && l.access == m) dup = true;
                    if (!dup) R.leaves.push_back({ch, m});
                }
            }
            R.order.push_back(id);
        };
        visit(root);
        return R;
    }

    // Emits the statements of a region; leaf values are named x<k>, the
    // accumulator `acc`; returns the name of the root value.
    std::string emit_region_body(const Region& R, std::ostringstream& o, const std::string& indent) {
        std::map<int, std::string> val;
        for (size_t k = 0; k < R.leaves.size(); ++k) {
            // a node may appear as FULL and ROW leaf; the FULL read names it
            if (!val.count(R.leaves[k].node) || R.leaves[k].access == FULL)
                val[R.leaves[k].node] = "x" + std::to_string(k);
        }
        if (R.acc >= 0) val[R.acc] = "acc";
        auto leafname = [&](int node, int m) {
            for (size_t k = 0; k < R.leaves.size(); ++k)
                if (R.leaves[k].node == node && R.leaves[k].access == m) return "x" + std::to_string(k);
            return val.at(node);
        };
        for (int id : R.order) {
            const Node& x = N(id);
            const int T = ct(id);
            std::string name = "t" + std::to_string(id);
            std::string e;
            auto arg = [&](int c) {
                int ch = x.ch[c];
                if (ch == R.acc) return std::string("acc");
                bool internal = ew[ch] && !mat[ch] && mode[id][c] == FULL;
                return internal ? val.at(ch) : leafname(ch, mode[id][c]);
            };
            auto binop = [&](const char* fn) {
                int ta = ct(x.ch[0]), tb = ct(x.ch[1]);
                int cm = common_type(ta, tb);
                return cast(T, cm, std::string("bafe::") + fn + "(" + cast(cm, ta, arg(0)) + ", " +
                                       cast(cm, tb, arg(1)) + ")");
            };
            switch (x.op) {
                case Op::Add: case Op::BiasAdd: e = binop("add"); break;
                case Op::Sub: e = binop("sub"); break;
                case Op::Mul: e = binop("mul"); break;
                case Op::FusedBiasRelu: e = "bafe::relu(" + binop("add") + ")"; break;
                case Op::Relu: e = "bafe::relu(" + cast(T, ct(x.ch[0]), arg(0)) + ")"; break;
                case Op::Neg: {
                    int tc = ct(x.ch[0]);
                    std::string ne = is_float(tc) ? "(-" + arg(0) + ")"
                                                  : std::string("bafe::sub((") + ctype(tc) + ")0, " + arg(0) + ")";
                    e = cast(T, tc, ne);
                    break;
                }
                case Op::Sigmoid: {
                    int tc = ct(x.ch[0]);
                    std::string ne = is_float(tc) ? "(-" + arg(0) + ")"
                                                  : std::string("bafe::sub((") + ctype(tc) + ")0, " + arg(0) + ")";
                    e = cast(T, BAFE_DTYPE_F32, "bafe::sigmoid_of_neg(" + cast(BAFE_DTYPE_F32, tc, ne) + ")");
                    break;
                }
                case Op::Tanh:
                    e = cast(T, BAFE_DTYPE_F32, "bafe::tanh_f(" + cast(BAFE_DTYPE_F32, ct(x.ch[0]), arg(0)) + ")");
                    break;
                case Op::Reshape: case Op::LayoutTransform:
                    e = cast(T, ct(x.ch[0]), arg(0));
                    break;
                default:
                    e = "0";
            }
            o << indent << "const " << ctype(T) << " " << name << " = " << e << ";\n";
            val[id] = name;
        }
        return val.at(R.root);
    }

    std::string kname(const char* what) {
        return std::string("bafe_") + what + "_s" + std::to_string(kcount++);
    }

    std::string describe_region(const Region& R) {
        std::function<std::string(int)> d = [&](int id) -> std::string {
            if (id == R.acc) return "acc";
            for (size_t k = 0; k < R.leaves.size(); ++k) {
                if (R.leaves[k].node != id) continue;
                bool internal = ew[id] && !mat[id];
                if (internal) break;
                const Node& x = N(id);
                std::string s = x.op == Op::Input ? x.name : ("%" + std::to_string(id));
                return R.leaves[k].access == ROW ? s + "[j]" : s;
            }
            const Node& x = N(id);
            std::string s = x.opname + "(";
            for (size_t c = 0; c < x.ch.size(); ++c) {
                if (c) s += ",";
                int ch = x.ch[c];
                bool internal = ew[ch] && !mat[ch] && mode[id][c] == FULL && ch != R.acc;
                if (internal || ch == R.acc) s += d(ch);
                else {
                    const Node& y = N(ch);
                    std::string nm = y.op == Op::Input ? y.name : ("%" + std::to_string(ch));
                    s += mode[id][c] == ROW ? nm + "[j]" : nm;
                }
            }
            return s + ")";
        };
        return d(R.root);
    }

    // Elementwise step for region R.
    int emit_ew(const Region& R) {
        Step s;
        s.kind = StepKind::Ew;
        s.dst = buf[R.root];
        const int root_store = buf_dtype[R.root];
        s.dst_esize = dtype_size(root_store);
        s.dst_bytes = N(R.root).shape.numel() * s.dst_esize;
        s.n = N(R.root).shape.numel();
        s.ncols = ncols_of(R.root);
        bool any_row = false;
        for (auto& l : R.leaves) {
            s.srcs.push_back(buf[l.node]);
            s.src_esize.push_back(dtype_size(buf_dtype[l.node]));
            s.src_row.push_back(l.access == ROW);
            any_row |= l.access == ROW;
        }
        s.kernel = kname("ew");
        s.kernel_vec = s.kernel + "_v4";
        const std::string P_ = "P_" + s.kernel, F_ = "f_" + s.kernel;
        src << "\n// step: " << describe_region(R) << "\n";
        src << "struct " << P_ << " {\n";
        for (size_t k = 0; k < R.leaves.size(); ++k)
            src << "  const " << dtype_ctype(buf_dtype[R.leaves[k].node]) << "* __restrict__ in" << k << ";\n";
        src << "  " << dtype_ctype(root_store) << "* __restrict__ out;\n  i64 n;\n  i64 ncols;\n};\n";
        src << "__device__ __forceinline__ " << dtype_ctype(root_store) << " " << F_ << "(";
        for (size_t k = 0; k < R.leaves.size(); ++k)
            src << (k ? ", " : "") << dtype_ctype(buf_dtype[R.leaves[k].node]) << " r" << k;
        src << ") {\n";
        for (size_t k = 0; k < R.leaves.size(); ++k) {
            int node = R.leaves[k].node;
            src << "  const " << ctype(ct(node)) << " x" << k << " = "
                << load_convert(buf_dtype[node], "r" + std::to_string(k)) << ";\n";
        }
        std::string rv = emit_region_body(R, src, "  ");
        src << "  return " << store_convert(root_store, ct(R.root), rv) << ";\n}\n";
        // scalar kernel
        src << "extern \"C\" __global__ void __launch_bounds__(256) " << s.kernel << "(const " << P_ << " p) {\n"
            << "  for (i64 i = (i64)blockIdx.x * blockDim.x + threadIdx.x; i < p.n; i += (i64)gridDim.x * blockDim.x) {\n";
        if (any_row) src << "    const i64 col = i % p.ncols;\n";
        src << "    p.out[i] = " << F_ << "(";
        for (size_t k = 0; k < R.leaves.size(); ++k)
            src << (k ? ", " : "") << "p.in" << k << "[" << (R.leaves[k].access == ROW ? "col" : "i") << "]";
        src << ");\n  }\n}\n";
        // 4-wide kernel (16-byte loads/stores); scalar tail in the same launch
        src << "extern \"C\" __global__ void __launch_bounds__(256) " << s.kernel_vec << "(const " << P_ << " p) {\n"
            << "  const i64 ng = p.n >> 2;\n"
            << "  const i64 step = (i64)gridDim.x * blockDim.x;\n"
            << "  i64 g = (i64)blockIdx.x * blockDim.x + threadIdx.x;\n";
        if (any_row) src << "  i64 col = (g << 2) % p.ncols;\n  const i64 dcol = (step << 2) % p.ncols;\n";
        src << "  for (; g < ng; g += step) {\n    const i64 e = g << 2;\n";
        for (size_t k = 0; k < R.leaves.size(); ++k)
            src << "    const auto v" << k << " = bafe::ld4(p.in" << k << " + " << (R.leaves[k].access == ROW ? "col" : "e") << ");\n";
        src << "    bafe::Vec4<" << dtype_ctype(root_store) << "> r;\n"
            << "#pragma unroll\n    for (int l = 0; l < 4; ++l) r.v[l] = " << F_ << "(";
        for (size_t k = 0; k < R.leaves.size(); ++k) src << (k ? ", " : "") << "v" << k << ".v[l]";
        src << ");\n    bafe::st4(p.out + e, r);\n";
        if (any_row) src << "    col += dcol; if (col >= p.ncols) col -= p.ncols;\n";
        src << "  }\n"
            << "  const i64 t = (i64)blockIdx.x * blockDim.x + threadIdx.x;\n"
            << "  const i64 i = (ng << 2) + t;\n"
            << "  if (t < 4 && i < p.n) {\n";
        if (any_row) src << "    const i64 c2 = i % p.ncols;\n";
        src << "    p.out[i] = " << F_ << "(";
        for (size_t k = 0; k < R.leaves.size(); ++k)
            src << (k ? ", " : "") << "p.in" << k << "[" << (R.leaves[k].access == ROW ? "c2" : "i") << "]";
        src << ");\n  }\n}\n";
        s.describe = "ew n=" + std::to_string((long long)s.n) + " " + dtype_ctype(root_store) + " " + describe_region(R) +
                     " -> " + bufname(s.dst);
        P.steps.push_back(s);
        return 0;
    }

    // Whether a GEMM operand is stored column-major.  Inputs carry BAFE's
    // layout tag (COL_MAJOR = Fortran buffer; BLOCKED / TENSOR_CORE data is
    // row-major, codegen.c:206-213 only tests COL_MAJOR).  Every buffer the
    // backend writes is row-major, so a transpose's output is read row-major
    // (the reference reads it column-major: wrong, see the defect list).
    bool col_storage(int id) const {
        const Node& x = N(id);
        if (x.op == Op::Input) return x.layout == BAFE_LAYOUT_COL_MAJOR;
        return false;
    }

    // GEMM step (optionally with region R as epilogue) for node gm.
    int emit_gemm(int gm, const Region* R) {
        const Node& g = N(gm);
        const Node& a = N(g.ch[0]);
        const Node& b = N(g.ch[1]);
        if (a.shape.rank < 2 || b.shape.rank < 2) { err = "matmul needs rank >= 2 operands"; return 2; }
        const int64_t M = g.shape.d[g.shape.rank - 2], Nn = g.shape.d[g.shape.rank - 1];
        const int64_t K = a.shape.d[a.shape.rank - 1];
        if (b.shape.d[b.shape.rank - 2] != K) {
            err = "matmul inner dimensions differ: " + a.shape.str() + " @ " + b.shape.str();
            return 2;
        }
        int64_t batch = 1;
        for (int d = 0; d < g.shape.rank - 2; ++d) batch *= g.shape.d[d];
        int64_t a_items = 1, b_items = 1;
        for (int d = 0; d < a.shape.rank - 2; ++d) a_items *= a.shape.d[d];
        for (int d = 0; d < b.shape.rank - 2; ++d) b_items *= b.shape.d[d];
        if ((a_items != batch && a_items != 1) || (b_items != batch && b_items != 1)) {
            err = "matmul batch dimensions do not match: " + a.shape.str() + " @ " + b.shape.str();
            return 2;
        }
        Step s;
        s.kind = StepKind::GemmExact;
        s.M = M; s.N = Nn; s.K = K; s.batch = batch;
        s.a_bstride = a_items == 1 ? 0 : M * K;
        s.b_bstride = b_items == 1 ? 0 : K * Nn;
        s.o_bstride = M * Nn;
        s.a_col = col_storage(g.ch[0]);
        s.b_col = col_storage(g.ch[1]);
        s.direct = g.op != Op::MatMul;
        s.srcs.push_back(buf[g.ch[0]]);
        s.srcs.push_back(buf[g.ch[1]]);
        const int root = R ? R->root : gm;
        s.dst = buf[root];
        const int out_store = buf_dtype[root];
        s.dst_esize = dtype_size(out_store);
        s.dst_bytes = N(root).shape.numel() * s.dst_esize;

        const int T = ct(gm);
        const int TA = compute_dtype(a.dtype), TB = compute_dtype(b.dtype);
        const int Pt = common_type(TA, TB), St = common_type(T, Pt);

        // Built-in epilogue of the fused forms (codegen.c:477-528): relu,
        // + bias[j], relu(+ bias[j]).  Its operand (bias) comes first.
        std::vector<Leaf> leaves;
        if (g.op == Op::FusedMatmulBias || g.op == Op::FusedMatmulBiasRelu) {
            if (g.ch.size() != 3 || N(g.ch[2]).shape.numel() != Nn || g.shape.rank != 2) {
                err = "fused_matmul_bias needs a rank-2 product and a bias of length N";
                return 2;
            }
            leaves.push_back({g.ch[2], ROW});
        }
        if (R) for (auto& l : R->leaves) leaves.push_back(l);
        if (leaves.size() > kEpilogueLeaves) { err = "GEMM epilogue reads more than 8 operands"; return 2; }

        // Tensor-core path choice.  f32 operands: tf32 MMAs (3xTF32 split by
        // default).  bf16 operands: kind::f16 MMAs -- the emitter converts
        // bf16 to f32 exactly (codegen.c:85-127) and bf16 x bf16 products are
        // exact in f32, so only the accumulation differs.  f16 operands stay
        // on the exact kernel: the emitter's f16 -> f32 conversion rescales
        // subnormals, which the tensor core would read as IEEE values.
        const std::string& prec = opt.gemm_precision;
        const bool f32_ops = T == BAFE_DTYPE_F32 && TA == BAFE_DTYPE_F32 && TB == BAFE_DTYPE_F32 &&
                             a.dtype == BAFE_DTYPE_F32 && b.dtype == BAFE_DTYPE_F32;
        const bool bf16_ops = T == BAFE_DTYPE_F32 && a.dtype == BAFE_DTYPE_BF16 && b.dtype == BAFE_DTYPE_BF16;
        if ((f32_ops || bf16_ops) && tc_shape_ok(s, f32_ops ? 4 : 2) && prec != "exact") {
            // auto: tensor cores from 256^3 multiply-adds on for bf16 (one
            // product per k-step), above 512^3 for f32 (three): up to there
            // the 3xTF32 plan (pre-passes + a few pair tiles) is latency-
            // bound and the bit-exact CUDA-core kernel, spread over enough
            // blocks, is faster (measured on B200, relu(A.B + C): 256^3 12.7
            // against 32.8 us, 512^3 35.6 against 38.9 us, 640^3 59.4
            // against 43.0 us)
            const double macs = (double)M * (double)Nn * (double)K;
            const bool big = bf16_ops ? macs >= 16777216.0 : macs > 134217728.0;   // 256^3 / 512^3
            if (prec == "tf32" || prec == "3xtf32" || big) {
                s.kind = StepKind::GemmTc;
                s.tc_variant = (bf16_ops || prec == "tf32") ? 1 : 3;
                s.tc_elem = bf16_ops ? 1 : 0;
                // 3xTF32 residuals: a pre-pass into plan scratch (default), or
                // made in shared memory by the kernel (tc_convert=1: no
                // scratch, half the operand traffic, more shared-memory
                // traffic).  With B split to nearest the in-kernel conversion
                // costs more than the two pre-pass launches even at 256^3
                // (32.9 against 24.8 us on B200; equal at 512^3, slower above),
                // so auto keeps the pre-pass.
                s.tc_convert = s.tc_variant == 3 && opt.tc_convert > 0;
                s.tc_pair = opt.tc_pair;
            }
        }

        s.kernel = kname(s.kind == StepKind::GemmTc ? "gemm_tc" : "gemm_exact");
        const std::string S_ = "Spec_" + s.kernel;
        std::string epi_desc = R ? describe_region(*R) : "acc";
        if (g.op == Op::FusedMatmulRelu) epi_desc = "relu(" + epi_desc + ")";
        if (g.op == Op::FusedMatmulBias) epi_desc = "add(" + epi_desc + "," + N(g.ch[2]).name + "[j])";
        if (g.op == Op::FusedMatmulBiasRelu) epi_desc = "relu(add(" + epi_desc + "," + N(g.ch[2]).name + "[j]))";
        src << "\n// step: " << g.opname << " " << a.shape.str() << " @ " << b.shape.str() << ", epilogue " << epi_desc << "\n";
        src << "struct " << S_ << " {\n"
            << "  typedef " << ctype(TA) << " TA;\n  typedef " << ctype(TB) << " TB;\n"
            << "  typedef " << ctype(T) << " T;\n  typedef " << ctype(Pt) << " P;\n  typedef " << ctype(St) << " S;\n"
            << "  typedef " << dtype_ctype(out_store) << " Out;\n"
            << "  static __device__ __forceinline__ TA loadA(const void* p, i64 i) { return "
            << load_convert(a.dtype, std::string("reinterpret_cast<const ") + dtype_ctype(a.dtype) + "*>(p)[i]") << "; }\n"
            << "  static __device__ __forceinline__ TB loadB(const void* p, i64 i) { return "
            << load_convert(b.dtype, std::string("reinterpret_cast<const ") + dtype_ctype(b.dtype) + "*>(p)[i]") << "; }\n";
        // apply(acc, g, b, i, j) -> the stored output element (i, j); and
        // apply4(acc4, g, b, i, j, o4): the same for columns j .. j+3 (j a
        // multiple of 4), each operand read as one 4-element vector (the
        // tensor-core kernels use it when every operand is aligned for that).
        // Both are the same statements; only the operand reads differ.
        auto emit_apply = [&](bool vec) {
            const std::string in = vec ? "      " : "    ";
            if (vec)
                src << "  template <class G> static __device__ __forceinline__ void apply4(const T* acc4, const G& g, i64 b, "
                       "i64 i, i64 j, bafe::Vec4<Out>& o4) {\n";
            else
                src << "  template <class G> static __device__ __forceinline__ Out apply(T acc_in, const G& g, i64 b, i64 i, i64 j) {\n";
            src << "    const i64 flat = b * g.o_bstride + i * g.N + j;\n    (void)flat;\n";
            // operand k of the epilogue (ep[k]) read at idx: the expression of
            // one element (inside apply4's loop: element e of its vector)
            auto operand = [&](int k, int node, const std::string& idx) {
                const std::string st = dtype_ctype(buf_dtype[node]);
                const std::string p = "reinterpret_cast<const " + st + "*>(g.ep[" + std::to_string(k) + "])";
                if (!vec) return p + "[" + idx + "]";
                src << "    const bafe::Vec4<" << st << "> v" << k << " = bafe::ld4(" << p << " + " << idx << ");\n";
                return "v" + std::to_string(k) + ".v[e]";
            };
            const bool bias = g.op == Op::FusedMatmulBias || g.op == Op::FusedMatmulBiasRelu;
            const int leaf_base = bias ? 1 : 0;
            std::string bias_rd;
            if (bias) bias_rd = operand(0, g.ch[2], "j");
            std::vector<std::string> leaf_rd;
            if (R)
                for (size_t k = 0; k < R->leaves.size(); ++k)
                    leaf_rd.push_back(operand(leaf_base + (int)k, R->leaves[k].node, R->leaves[k].access == ROW ? "j" : "flat"));
            if (vec) src << "#pragma unroll\n    for (int e = 0; e < 4; ++e) {\n" << in << "const T acc_in = acc4[e];\n";
            // built-in epilogue first
            std::string accexpr = "acc_in";
            if (g.op == Op::FusedMatmulRelu) {
                src << in << "const T acc0 = bafe::relu(acc_in);\n";
                accexpr = "acc0";
            } else if (bias) {
                const int tb = ct(g.ch[2]);
                const int cm = common_type(T, tb);
                src << in << "const " << ctype(tb) << " bias = " << load_convert(buf_dtype[g.ch[2]], bias_rd) << ";\n";
                std::string sum = cast(T, cm, "bafe::add(" + cast(cm, T, "acc_in") + ", " + cast(cm, tb, "bias") + ")");
                if (g.op == Op::FusedMatmulBiasRelu) sum = "bafe::relu(" + sum + ")";
                src << in << "const T acc0 = " << sum << ";\n";
                accexpr = "acc0";
            }
            src << in << "const T acc = " << accexpr << ";\n" << in << "(void)acc;\n";
            std::string rv = "acc";
            int rv_dtype = T;
            if (R) {
                for (size_t k = 0; k < R->leaves.size(); ++k)
                    src << in << "const " << ctype(ct(R->leaves[k].node)) << " x" << k << " = "
                        << load_convert(buf_dtype[R->leaves[k].node], leaf_rd[k]) << ";\n";
                rv = emit_region_body(*R, src, in);
                rv_dtype = ct(R->root);
            }
            if (vec) src << in << "o4.v[e] = " << store_convert(out_store, rv_dtype, rv) << ";\n    }\n  }\n";
            else src << "    return " << store_convert(out_store, rv_dtype, rv) << ";\n  }\n";
        };
        emit_apply(false);
        emit_apply(true);
        // prefetch(g, b, i, j0): row i, columns j0 .. j0+127 of every
        // full-size epilogue operand into L2 (bounds-checked, a hint), so
        // the epilogue's loads after the tile's last chunk find them there
        // (row-vector operands are small and stay cached anyway).
        src << "  template <class G> static __device__ __forceinline__ void prefetch(const G& g, i64 b, i64 i, i64 j0) {\n"
            << "    if (i >= g.M) return;\n    (void)b; (void)j0;\n";
        if (R) {
            const int leaf_base = (g.op == Op::FusedMatmulBias || g.op == Op::FusedMatmulBiasRelu) ? 1 : 0;
            for (size_t k = 0; k < R->leaves.size(); ++k) {
                if (R->leaves[k].access == ROW) continue;
                const int es = dtype_size(buf_dtype[R->leaves[k].node]);
                const int per_line = 128 / es;
                src << "    for (int l = 0; l < " << (128 + per_line - 1) / per_line << "; ++l) {\n"
                    << "      const i64 j = j0 + l * " << per_line << ";\n"
                    << "      if (j < g.N) bafe::prefetch_l2(reinterpret_cast<const char*>(g.ep[" << leaf_base + (int)k
                    << "]) + (b * g.o_bstride + i * g.N + j) * " << es << ");\n    }\n";
            }
        }
        src << "  }\n";
        src << "};\n";
        for (auto& l : leaves) s.srcs.push_back(buf[l.node]);
        s.n_epi = (int)leaves.size();
        s.src_esize = {dtype_size(buf_dtype[g.ch[0]]), dtype_size(buf_dtype[g.ch[1]])};
        s.src_row = {false, false};
        for (auto& l : leaves) {
            s.src_esize.push_back(dtype_size(buf_dtype[l.node]));
            s.src_row.push_back(l.access == ROW);
        }
        if (s.kind == StepKind::GemmTc && s.tc_variant == 3 && !s.tc_convert) {
            // 3xTF32 operand parts, written once per call by streaming
            // pre-passes into plan scratch: A split to nearest, A_lo and A_hi
            // (bafe::tf32_split); B_lo = rn_tf32(x - trunc_tf32(x)) (B's raw
            // values are its hi part, truncated by the tensor core).  One
            // operand rounded to nearest keeps the dropped lo.lo term free
            // of the product's sign; rounding A -- a row panel per rank when
            // the GEMM is sharded -- rather than B, which every rank reads
            // whole, leaves each rank one write of B instead of two.
            // aux = {A_lo, B_lo, A_hi}.
            BufRef a_hi;
            s.aux.push_back(emit_residual(s.srcs[0], M * K * a_items, "A", &a_hi));
            s.aux.push_back(emit_residual(s.srcs[1], K * Nn * b_items, "B"));
            s.aux.push_back(a_hi);
        }
        if (s.kind == StepKind::GemmExact) {
            // the widest micro-tile that still gives >= 128 blocks (a
            // 64x64 tile per block leaves most SMs idle on small problems)
            s.exact_tm = 4;
            auto blocks = [&](int64_t t) { return ((M + t - 1) / t) * ((Nn + t - 1) / t) * std::max<int64_t>(batch, 1); };
            while (s.exact_tm > 1 && blocks(16 * s.exact_tm) < 128) s.exact_tm /= 2;
            src << "extern \"C\" __global__ void __launch_bounds__(256) " << s.kernel
                << "(const bafe::GemmArgs g) { bafe::gemm_exact<" << S_ << ", " << (s.direct ? "true" : "false")
                << ", " << s.exact_tm << ">(g); }\n";
        } else {
            const char* cfg = s.tc_pair ? "TcPairCfg" : "TcCfg";
            const char* fn = s.tc_pair ? "gemm_tc_pair" : "gemm_tc";
            const char* elem = s.tc_elem == 1 ? "bafe::ElemBf16" : "bafe::ElemTf32";
            src << "extern \"C\" __global__ void __launch_bounds__(bafe::" << cfg << "<" << s.tc_variant
                << ">::THREADS, 1) " << s.kernel << "(const __grid_constant__ bafe::TcArgs g) { bafe::" << fn << "<"
                << S_ << ", " << s.tc_variant << ", " << elem << ", " << (s.tc_convert ? "true" : "false")
                << ">(g); }\n";
            // the partial sums of split tail tiles -> epilogue (launched only when the tail splits)
            s.kernel_vec = s.kernel + "_fix";
            src << "extern \"C\" __global__ void __launch_bounds__(256) " << s.kernel_vec
                << "(const __grid_constant__ bafe::TcArgs g) { bafe::gemm_tc_fixup<" << S_ << ", "
                << (s.tc_pair ? 256 : 128) << ">(g); }\n";
        }
        char geo[256];
        snprintf(geo, sizeof(geo), " batch=%lld m=%lld n=%lld k=%lld a=%s b=%s", (long long)batch, (long long)M,
                 (long long)Nn, (long long)K, s.a_col ? "col" : "row", s.b_col ? "col" : "row");
        std::string kindname = s.kind == StepKind::GemmTc ? std::string(s.tc_elem == 1 ? "gemm.tc.bf16"
                                                                        : s.tc_variant == 1 ? "gemm.tc.tf32" : "gemm.tc.3xtf32") +
                                                                (s.tc_pair ? ".pair" : "")
                                                          : (s.direct ? "gemm.exact.direct" : "gemm.exact.chunk32");
        if (s.kind == StepKind::GemmExact) kindname += " tile=" + std::to_string(16 * s.exact_tm);
        s.describe = kindname + geo + " epi=" + epi_desc + " -> " + bufname(s.dst);
        P.steps.push_back(s);
        return 0;
    }

    // The tensor-core kernel reads A and B through TMA: row strides (and
    // with them the per-batch strides) must be multiples of 16 bytes.
    bool tc_shape_ok(const Step& s, int esize) const {
        if (!tc_available()) return false;
        if (s.batch < 1 || s.batch > (1 << 20)) return false;
        if (s.M < 1 || s.N < 1 || s.K < 1) return false;
        // tile origins and TMA coordinates are 32-bit, tile indices too
        const int64_t lim = (int64_t(1) << 31) - 1024;
        if (s.M > lim || s.N > lim || s.K > lim) return false;
        if (((s.M + 255) / 256) * ((s.N + 255) / 256) * s.batch > lim) return false;
        const int64_t a_ld = s.a_col ? s.M : s.K;
        const int64_t b_ld = s.b_col ? s.K : s.N;
        if ((a_ld * esize) % 16 || (b_ld * esize) % 16) return false;
        if (s.N % 4) return false;   // vectorised epilogue
        return true;
    }
    static bool tc_available();

    // Streaming pre-pass over an f32 buffer: writes its tf32 residual
    // (bafe::tf32_lo: the raw values stay the hi part) or, when hi_out is
    // given, its round-to-nearest split (bafe::tf32_split): lo to the step's
    // output, hi to a second output.
    BufRef emit_residual(const BufRef& from, int64_t n, const char* what, BufRef* hi_out = nullptr) {
        Step s;
        s.kind = StepKind::Ew;
        s.n = n;
        s.ncols = 1;
        s.dst = new_tmp(n * 4);
        s.dst_esize = 4;
        s.dst_bytes = n * 4;
        if (hi_out) {
            s.dst2 = new_tmp(n * 4);
            s.has_dst2 = true;
            *hi_out = s.dst2;
        }
        s.srcs.push_back(from);
        s.src_esize.push_back(4);
        s.src_row.push_back(false);
        s.kernel = kname(hi_out ? "tf32_split" : "tf32_residual");
        s.kernel_vec = s.kernel + "_v4";
        // per element: hi (split only) and lo of x
        auto body = [&](const std::string& x, const std::string& hi, const std::string& lo) -> std::string {
            if (!hi_out) return lo + " = bafe::tf32_lo(" + x + ");";
            return "{ float h_, l_; bafe::tf32_split(" + x + ", h_, l_); " + hi + " = h_; " + lo + " = l_; }";
        };
        src << "\nstruct P_" << s.kernel << " { const float* __restrict__ in0; float* __restrict__ out; i64 n; i64 ncols;"
            << (hi_out ? " float* __restrict__ out2;" : "") << " };\n"
            << "extern \"C\" __global__ void __launch_bounds__(256) " << s.kernel << "(const P_" << s.kernel << " p) {\n"
            << "  for (i64 i = (i64)blockIdx.x * blockDim.x + threadIdx.x; i < p.n; i += (i64)gridDim.x * blockDim.x)\n"
            << "    " << body("p.in0[i]", "p.out2[i]", "p.out[i]") << "\n}\n"
            << "extern \"C\" __global__ void __launch_bounds__(256) " << s.kernel_vec << "(const P_" << s.kernel << " p) {\n"
            << "  const i64 ng = p.n >> 2;\n"
            << "  for (i64 g = (i64)blockIdx.x * blockDim.x + threadIdx.x; g < ng; g += (i64)gridDim.x * blockDim.x) {\n"
            << "    const auto v = bafe::ld4(p.in0 + 4 * g);\n    bafe::Vec4<float> r, rh;\n"
            << "#pragma unroll\n    for (int l = 0; l < 4; ++l) " << body("v.v[l]", "rh.v[l]", "r.v[l]") << "\n"
            << "    bafe::st4(p.out + 4 * g, r);\n"
            << (hi_out ? "    bafe::st4(p.out2 + 4 * g, rh);\n" : "") << "  }\n"
            << "  const i64 t = (i64)blockIdx.x * blockDim.x + threadIdx.x;\n"
            << "  if (t < 4 && (ng << 2) + t < p.n) "
            << body("p.in0[(ng << 2) + t]", "p.out2[(ng << 2) + t]", "p.out[(ng << 2) + t]") << "\n}\n";
        s.describe = std::string("ew n=") + std::to_string((long long)n) + " float " +
                     (hi_out ? "tf32_split(" : "tf32_residual(") + what + ") -> " + bufname(s.dst) +
                     (hi_out ? " (lo), " + bufname(s.dst2) + " (hi)" : "");
        P.steps.push_back(s);
        return s.dst;
    }

    // Converts a half-precision buffer to f32 for steps that read compute
    // types only (transpose, gather, reduce).
    BufRef as_compute(int node) {
        if (buf_dtype[node] != BAFE_DTYPE_F16 && buf_dtype[node] != BAFE_DTYPE_BF16) return buf[node];
        Region R;
        R.root = -1;
        Step s;
        s.kind = StepKind::Ew;
        s.n = N(node).shape.numel();
        s.ncols = 1;
        s.dst = new_tmp(s.n * 4);
        s.dst_esize = 4;
        s.dst_bytes = s.n * 4;
        s.srcs.push_back(buf[node]);
        s.src_esize.push_back(2);
        s.src_row.push_back(false);
        s.kernel = kname("cvt");
        s.kernel_vec = s.kernel + "_v4";
        const char* conv = buf_dtype[node] == BAFE_DTYPE_F16 ? "bafe::f16_to_f32" : "bafe::bf16_to_f32";
        src << "\nstruct P_" << s.kernel << " { const u16* __restrict__ in0; float* __restrict__ out; i64 n; i64 ncols; };\n"
            << "extern \"C\" __global__ void __launch_bounds__(256) " << s.kernel << "(const P_" << s.kernel << " p) {\n"
            << "  for (i64 i = (i64)blockIdx.x * blockDim.x + threadIdx.x; i < p.n; i += (i64)gridDim.x * blockDim.x)\n"
            << "    p.out[i] = " << conv << "(p.in0[i]);\n}\n"
            << "extern \"C\" __global__ void __launch_bounds__(256) " << s.kernel_vec << "(const P_" << s.kernel << " p) {\n"
            << "  for (i64 i = (i64)blockIdx.x * blockDim.x + threadIdx.x; i < p.n; i += (i64)gridDim.x * blockDim.x)\n"
            << "    p.out[i] = " << conv << "(p.in0[i]);\n}\n";
        s.describe = std::string("convert ") + (buf_dtype[node] == BAFE_DTYPE_F16 ? "f16" : "bf16") + "->f32 n=" +
                     std::to_string((long long)s.n);
        P.steps.push_back(s);
        return s.dst;
    }

    // Writes a compute-typed temporary into the half-typed output.
    void emit_store_convert(BufRef from, int node) {
        Step s;
        s.kind = StepKind::Ew;
        s.n = N(node).shape.numel();
        s.ncols = 1;
        s.dst = buf[node];
        s.dst_esize = 2;
        s.dst_bytes = s.n * 2;
        s.srcs.push_back(from);
        s.src_esize.push_back(4);
        s.src_row.push_back(false);
        s.kernel = kname("cvt");
        s.kernel_vec = s.kernel + "_v4";
        const char* conv = buf_dtype[node] == BAFE_DTYPE_F16 ? "bafe::f32_to_f16" : "bafe::f32_to_bf16";
        src << "\nstruct P_" << s.kernel << " { const float* __restrict__ in0; u16* __restrict__ out; i64 n; i64 ncols; };\n"
            << "extern \"C\" __global__ void __launch_bounds__(256) " << s.kernel << "(const P_" << s.kernel << " p) {\n"
            << "  for (i64 i = (i64)blockIdx.x * blockDim.x + threadIdx.x; i < p.n; i += (i64)gridDim.x * blockDim.x)\n"
            << "    p.out[i] = " << conv << "(p.in0[i]);\n}\n"
            << "extern \"C\" __global__ void __launch_bounds__(256) " << s.kernel_vec << "(const P_" << s.kernel << " p) {\n"
            << "  for (i64 i = (i64)blockIdx.x * blockDim.x + threadIdx.x; i < p.n; i += (i64)gridDim.x * blockDim.x)\n"
            << "    p.out[i] = " << conv << "(p.in0[i]);\n}\n";
        s.describe = "convert f32->half n=" + std::to_string((long long)s.n);
        P.steps.push_back(s);
    }

    // Destination of a compute-typed step writing node `id`'s value.
    BufRef compute_dst(int id, bool& needs_store_convert) {
        needs_store_convert = false;
        if (id == G.root && (buf_dtype[id] == BAFE_DTYPE_F16 || buf_dtype[id] == BAFE_DTYPE_BF16)) {
            needs_store_convert = true;
            return new_tmp(N(id).shape.numel() * 4);
        }
        return buf[id];
    }

    int emit_transpose(int id) {
        const Node& x = N(id);
        const Node& c = N(x.ch[0]);
        const int T = ct(id);
        BufRef in = as_compute(x.ch[0]);
        bool conv;
        BufRef dst = compute_dst(id, conv);
        Step s;
        s.srcs.push_back(in);
        s.dst = dst;
        s.dst_esize = dtype_size(T);
        s.dst_bytes = x.shape.numel() * s.dst_esize;
        const char* ty = ctype(T);
        // rank >= 3 with the last two axes swapped and the others in place:
        // a batch of rank-2 transposes (self-inverse, so the emitter's own
        // rank-N indexing, codegen.c:371-404, agrees)
        bool batched2d = x.shape.rank >= 3 && c.shape.rank == x.shape.rank && (int)x.perm.size() == x.shape.rank;
        for (int d = 0; batched2d && d < x.shape.rank - 2; ++d) batched2d = x.perm[d] == d;
        batched2d = batched2d && x.perm[x.shape.rank - 2] == x.shape.rank - 1 && x.perm[x.shape.rank - 1] == x.shape.rank - 2;
        if ((x.shape.rank == 2 && c.shape.rank == 2) || batched2d) {
            // codegen.c:363-369: out (M,N), out[i*N+j] = x[j*M+i], per batch item
            const int R2 = x.shape.rank;
            s.kind = StepKind::Transpose2d;
            s.M = x.shape.d[R2 - 2];
            s.N = x.shape.d[R2 - 1];
            s.batch = 1;
            for (int d = 0; d < R2 - 2; ++d) s.batch *= x.shape.d[d];
            s.kernel = kname("transpose");
            src << "\nextern \"C\" __global__ void __launch_bounds__(256) " << s.kernel << "(const " << ty << "* x, " << ty
                << "* out, i64 M, i64 N, i64 ldx) { bafe::transpose2d<" << ty << ">(x, out, M, N, ldx); }\n";
            if (dtype_size(T) == 4) {
                s.kernel_vec = s.kernel + "_v4";
                src << "extern \"C\" __global__ void __launch_bounds__(256) " << s.kernel_vec << "(const " << ty
                    << "* x, " << ty << "* out, i64 M, i64 N, i64 ldx) { bafe::transpose2d_w4<" << ty
                    << ">(x, out, M, N, ldx); }\n";
            }
            s.describe = "transpose2d m=" + std::to_string((long long)s.M) + " n=" + std::to_string((long long)s.N) +
                         (s.batch > 1 ? " batch=" + std::to_string((long long)s.batch) : std::string());
        } else {
            // Rank-N: out[o] = x[i] with i_{perm[d]} = o_d.  The emitter's
            // own rank-N indexing (codegen.c:371-404) is only right for
            // self-inverse permutations; this is the correct transpose and
            // coincides with the reference wherever the reference is right.
            const int R = x.shape.rank;
            if ((int)x.perm.size() != R || c.shape.rank != R) { err = "transpose perm does not match the rank"; return 2; }
            int64_t istride[8];
            for (int d = R - 1; d >= 0; --d) istride[d] = (d == R - 1) ? 1 : istride[d + 1] * c.shape.d[d + 1];
            s.kind = StepKind::Gather;
            s.grank = R;
            for (int d = 0; d < R; ++d) {
                int p = x.perm[d];
                if (p < 0 || p >= R) { err = "transpose perm out of range"; return 2; }
                s.gdims[d] = x.shape.d[d];
                s.gstride[d] = istride[p];
            }
            s.n = x.shape.numel();
            s.kernel = kname("gather");
            src << "\nextern \"C\" __global__ void __launch_bounds__(256) " << s.kernel << "(const " << ty << "* x, " << ty
                << "* out, const bafe::GatherArgs g) { bafe::gather_nd<" << ty << ">(x, out, g); }\n";
            emit_gather_v4(s, ty);
            s.describe = "transpose rank " + std::to_string(R) + " n=" + std::to_string((long long)s.n);
        }
        P.steps.push_back(s);
        if (conv) emit_store_convert(dst, id);
        return 0;
    }

    // The vector entry of a gather step (kernel_vec), when its innermost axis
    // reads contiguous, 4-aligned runs of x (gather_nd_v4).
    void emit_gather_v4(Step& s, const char* ty) {
        const int R = s.grank;
        if (R < 1 || s.gstride[R - 1] != 1 || s.gdims[R - 1] % 4 != 0) return;
        for (int d = 0; d < R - 1; ++d)
            if (s.gstride[d] % 4 != 0) return;
        s.kernel_vec = s.kernel + "_v4";
        src << "extern \"C\" __global__ void __launch_bounds__(256) " << s.kernel_vec << "(const " << ty << "* x, " << ty
            << "* out, const bafe::GatherArgs g) { bafe::gather_nd_v4<" << ty << ">(x, out, g); }\n";
    }

    int emit_broadcast(int id) {
        // numpy broadcasting of the child to attrs.shape.  (The emitter
        // memcpy's numel(out) bytes from the smaller buffer, codegen.c:465,
        // reading out of range; this is the intended semantics.)
        const Node& x = N(id);
        const Node& c = N(x.ch[0]);
        const int T = ct(id);
        BufRef in = as_compute(x.ch[0]);
        bool conv;
        BufRef dst = compute_dst(id, conv);
        const int R = x.shape.rank;
        if (c.shape.rank > R) { err = "broadcast_to to a lower rank"; return 2; }
        Step s;
        s.kind = StepKind::Gather;
        s.srcs.push_back(in);
        s.dst = dst;
        s.dst_esize = dtype_size(T);
        s.dst_bytes = x.shape.numel() * s.dst_esize;
        s.grank = R;
        int64_t st = 1;
        for (int d = R - 1; d >= 0; --d) {
            int cd = d - (R - c.shape.rank);
            int64_t cdim = cd >= 0 ? c.shape.d[cd] : 1;
            if (cdim != 1 && cdim != x.shape.d[d]) { err = "broadcast_to: incompatible shapes " + c.shape.str() + " -> " + x.shape.str(); return 2; }
            s.gdims[d] = x.shape.d[d];
            s.gstride[d] = (cdim == 1) ? 0 : st;
            if (cd >= 0) st *= cdim;
        }
        s.n = x.shape.numel();
        s.kernel = kname("broadcast");
        const char* ty = ctype(T);
        src << "\nextern \"C\" __global__ void __launch_bounds__(256) " << s.kernel << "(const " << ty << "* x, " << ty
            << "* out, const bafe::GatherArgs g) { bafe::gather_nd<" << ty << ">(x, out, g); }\n";
        emit_gather_v4(s, ty);
        s.describe = "broadcast_to " + c.shape.str() + " -> " + x.shape.str();
        P.steps.push_back(s);
        if (conv) emit_store_convert(dst, id);
        return 0;
    }

    int emit_reduce(int id) {
        const Node& x = N(id);
        const Node& c = N(x.ch[0]);
        const int T = ct(id);
        bool conv;
        BufRef dst = compute_dst(id, conv);
        Step s;
        s.dst = dst;
        s.dst_esize = dtype_size(T);
        s.dst_bytes = x.shape.numel() * s.dst_esize;
        const bool is_max = x.op == Op::ReduceMax;
        if (x.axes.size() == 1 && (c.shape.rank == 1 || c.shape.rank == 2)) {
            BufRef in = as_compute(x.ch[0]);
            s.kind = StepKind::Reduce;
            s.srcs.push_back(in);
            if (c.shape.rank == 1) { s.M = 1; s.N = c.shape.d[0]; s.axis = 1; }
            else { s.M = c.shape.d[0]; s.N = c.shape.d[1]; s.axis = (x.axes[0] % 2) == 0 ? 0 : 1; }
            s.kernel = kname(is_max ? "reduce_max" : "reduce_sum");
            const char* ty = ctype(T);
            src << "\nextern \"C\" __global__ void __launch_bounds__(256) " << s.kernel << "(const " << ty << "* x, " << ty
                << "* out, i64 M, i64 N, int axis) { bafe::reduce_axis<" << ty << ", " << (is_max ? "true" : "false")
                << ">(x, out, M, N, axis); }\n";
            s.describe = std::string(is_max ? "reduce_max" : "reduce_sum") + " m=" + std::to_string((long long)s.M) +
                         " n=" + std::to_string((long long)s.N) + " axis=" + std::to_string(s.axis);
        } else {
            // The emitter's generic reduce zero-fills (codegen.c:446-451).
            s.kind = StepKind::Zero;
            s.describe = "zero-fill (multi-axis reduce is a zero-filling TODO in the reference)";
        }
        P.steps.push_back(s);
        if (conv) emit_store_convert(dst, id);
        return 0;
    }

    // ---------------------------------------------------------- schedule --
    int run() {
        if (int rc = analyse()) return rc;
        assign_buffers();
        P.n_inputs = (int)G.inputs.size();
        for (int id : G.inputs) {
            P.in_dtypes.push_back(N(id).dtype);
            P.in_bytes.push_back(N(id).shape.numel() * dtype_size(N(id).dtype));
        }
        src << "#include \"bafe_dev.cuh\"\n#include \"layout.cuh\"\n#include \"gemm_exact.cuh\"\n"
               "#include \"gemm_tc.cuh\"\n";
        // Post-order walk from the root: every materialised node becomes a
        // step after its producers.
        std::vector<char> done(G.nodes.size(), 0);
        std::function<int(int)> need = [&](int id) -> int {
            if (done[id]) return 0;
            done[id] = 1;
            const Node& x = N(id);
            if (x.op == Op::Input) return 0;
            if (ew[id] && !mat[id]) {
                for (size_t c = 0; c < x.ch.size(); ++c)
                    if (int rc = need(x.ch[c])) return rc;
                return 0;
            }
            if (is_gemm_op(x.op) && fused_into[id] >= 0) {
                for (int c : x.ch) if (int rc = need(c)) return rc;
                return 0;
            }
            for (int c : x.ch) if (int rc = need(c)) return rc;
            if (ew[id]) {
                Region R = collect_region(id);
                if (R.acc >= 0) return emit_gemm(R.acc, &R);
                if (R.leaves.size() > kRegionLeaves) { err = "elementwise region reads more than 16 operands"; return 2; }
                return emit_ew(R);
            }
            switch (x.op) {
                case Op::MatMul: case Op::FusedMatmulRelu: case Op::FusedMatmulBias: case Op::FusedMatmulBiasRelu:
                    if (x.op == Op::FusedMatmulRelu && x.ch.size() != 2) { err = "fused_matmul_relu arity"; return 2; }
                    return emit_gemm(id, nullptr);
                case Op::Transpose: return emit_transpose(id);
                case Op::BroadcastTo: return emit_broadcast(id);
                case Op::ReduceSum: case Op::ReduceMax: return emit_reduce(id);
                default: {
                    // Unknown op (e.g. "scale"): the emitter zero-fills the
                    // node's buffer (codegen.c:529-533); so do we.
                    Step s;
                    s.kind = StepKind::Zero;
                    s.dst = buf[id];
                    s.dst_esize = dtype_size(buf_dtype[id]);
                    s.dst_bytes = x.shape.numel() * s.dst_esize;
                    s.describe = "zero-fill (unsupported op '" + x.opname + "', as the reference emitter does)";
                    P.steps.push_back(s);
                    return 0;
                }
            }
        };
        if (int rc = need(G.root)) return rc;
        // The root may be an input (f(x) = x) or an alias of one: copy it
        // through an identity region.
        if (N(G.root).op == Op::Input) {
            Step s;
            s.kind = StepKind::Ew;
            s.n = N(G.root).shape.numel();
            s.ncols = 1;
            s.dst = {BufRef::Out, 0};
            s.dst_esize = dtype_size(N(G.root).dtype);
            s.dst_bytes = P.out_bytes;
            BufRef in{BufRef::In, N(G.root).input_index};
            s.srcs.push_back(in);
            s.src_esize.push_back(dtype_size(N(G.root).dtype));
            s.src_row.push_back(false);
            s.kernel = kname("copy");
            s.kernel_vec = s.kernel + "_v4";
            const char* ty = dtype_ctype(N(G.root).dtype);
            // f16 inputs round-trip through the emitter's conversions
            std::string val = "p.in0[i]";
            if (N(G.root).dtype == BAFE_DTYPE_F16) val = "bafe::f32_to_f16(bafe::f16_to_f32(p.in0[i]))";
            if (N(G.root).dtype == BAFE_DTYPE_BF16) val = "bafe::f32_to_bf16(bafe::bf16_to_f32(p.in0[i]))";
            src << "\nstruct P_" << s.kernel << " { const " << ty << "* __restrict__ in0; " << ty
                << "* __restrict__ out; i64 n; i64 ncols; };\n"
                << "extern \"C\" __global__ void __launch_bounds__(256) " << s.kernel << "(const P_" << s.kernel << " p) {\n"
                << "  for (i64 i = (i64)blockIdx.x * blockDim.x + threadIdx.x; i < p.n; i += (i64)gridDim.x * blockDim.x)\n"
                << "    p.out[i] = " << val << ";\n}\n"
                << "extern \"C\" __global__ void __launch_bounds__(256) " << s.kernel_vec << "(const P_" << s.kernel << " p) {\n"
                << "  for (i64 i = (i64)blockIdx.x * blockDim.x + threadIdx.x; i < p.n; i += (i64)gridDim.x * blockDim.x)\n"
                << "    p.out[i] = " << val << ";\n}\n";
            s.describe = "copy input -> out n=" + std::to_string((long long)s.n);
            P.steps.push_back(s);
        }
        P.source = src.str();
        P.source_hash = sha256_hex(P.source.data(), P.source.size());
        std::ostringstream d;
        for (auto& s : P.steps) d << s.describe << "\n";
        P.describe = d.str();
        analyse_row_streaming(P, N(G.root).shape);
        return 0;
    }
};

}  // namespace

bool tc_kernel_enabled();

bool Lowerer::tc_available() { return tc_kernel_enabled(); }

int lower_graph(const Graph& g, const Options& opt, Plan& plan, std::string& err) {
    Lowerer L(g, opt, plan, err);
    return L.run();
}

}  // namespace bafe_cuda
