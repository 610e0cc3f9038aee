// streaming.cpp -- which parts of a plan split by output row.
//
// A host call of a plan (the reference's kernel ABI: host pointers in,
// host pointer out) moves every input over PCIe, runs the kernels and moves
// the output back.  Done in that order the copies and the kernels add up.
// When the plan's work is row-separable -- each output row depends only on
// the same rows of some inputs and on the whole of the others -- the call
// can instead stream row panels: copy panel p's rows while the kernels work
// on panel p-1 and the output rows of panel p-2 travel back.  The host-to-
// device link is then the only serial cost.
//
// The analysis walks the steps from the last to the first, starting from
// the output (split, one row per output row):
//   * a step whose destination is split runs once per panel:
//       - elementwise: n = rows * e elements; full-shape operands split with
//         e elements per row, row-vector operands (index i % ncols) stay
//         whole (e must be a multiple of ncols);
//       - GEMM (batch 1, M = rows): A splits with K elements per row (A must
//         be row-major so a panel is contiguous), B stays whole, epilogue
//         operands split with N per row (full) or stay whole (row vector);
//         the 3xTF32 residual of A splits like A, the parts of B (lo, hi)
//         stay whole; an elementwise step with a second output writes it
//         row for row with its first;
//   * a step whose destination is whole runs once, before the panels, and
//     needs every operand whole;
//   * any other step kind with a split destination, or a buffer needed both
//     split and whole, or split with two different row sizes, makes the
//     plan not streamable (host calls then run it in one piece).
#include "internal.h"

#include <map>
#include <utility>

namespace bafe_cuda {

// A plan that is exactly one rank-2 transpose, input 0 -> output (out (M, N),
// out[i][j] = x[j][i]): output rows [r0, r1) are x's columns [r0, r1), one
// element of every x row per output row.  The host call streams it like a
// row-split plan, copying each panel's band of columns with one strided
// copy, so the input and output copies run at the same time.
static void analyse_column_streaming(Plan& P, int64_t R) {
    P.stream_cols = false;
    if (P.steps.size() != 1 || P.n_inputs != 1) return;
    Step& s = P.steps[0];
    if (s.kind != StepKind::Transpose2d || s.batch != 1 || s.M != R || s.M < 2 || s.N < 1) return;
    if (s.srcs.size() != 1 || s.srcs[0].kind != BufRef::In || s.srcs[0].idx != 0 || s.dst.kind != BufRef::Out) return;
    if (s.dst_esize <= 0 || P.in_bytes[0] != s.M * s.N * s.dst_esize) return;
    s.panel = true;
    s.dst_rb = s.N * s.dst_esize;          // output: whole rows
    s.src_rb.assign(1, s.dst_esize);       // input: r0 columns in
    P.in_rb[0] = s.N * s.dst_esize;        // bytes per output row, moved by the strided copy
    P.out_rb = s.N * s.dst_esize;
    P.stream_rows = R;
    P.stream_align = 64;                   // whole 64 x 64 tiles, 16-byte aligned column offsets
    P.stream_cols = true;
}

void analyse_row_streaming(Plan& P, const Shape& out_shape) {
    P.stream_cols = false;
    P.stream_ok = false;
    P.stream_rows = 0;
    P.in_rb.assign(P.n_inputs, 0);
    P.out_rb = 0;
    for (auto& s : P.steps) {
        s.panel = false;
        s.row_elems = 0;
        s.dst_rb = 0;
        s.src_rb.assign(s.srcs.size(), 0);
        s.aux_rb.assign(s.aux.size(), 0);
    }
    if (out_shape.rank < 1 || P.out_bytes <= 0 || P.steps.empty()) return;
    const int64_t R = out_shape.d[0];
    if (R < 2 || P.out_bytes % R) return;

    // bytes per row of each buffer; absent = not yet needed
    std::map<std::pair<int, int>, int64_t> rb;
    bool ok = true;
    auto key = [](const BufRef& b) { return std::make_pair((int)b.kind, b.kind == BufRef::Out ? 0 : b.idx); };
    auto need = [&](const BufRef& b, int64_t bytes) {
        auto k = key(b);
        auto it = rb.find(k);
        if (it == rb.end()) rb[k] = bytes;
        else if (it->second != bytes) ok = false;
    };
    rb[{(int)BufRef::Out, 0}] = P.out_bytes / R;

    for (int si = (int)P.steps.size() - 1; si >= 0 && ok; --si) {
        Step& s = P.steps[si];
        auto it = rb.find(key(s.dst));
        const int64_t drb = it == rb.end() ? 0 : it->second;
        if (drb == 0) {   // runs once per call: every operand whole
            for (auto& b : s.srcs) need(b, 0);
            for (auto& b : s.aux) need(b, 0);
            if (s.has_dst2) need(s.dst2, 0);
            continue;
        }
        s.panel = true;
        s.dst_rb = drb;
        switch (s.kind) {
            case StepKind::Ew: {
                if (s.has_dst2) need(s.dst2, drb);   // written row for row with dst
                if (s.n % R) { ok = false; break; }
                const int64_t e = s.n / R;
                if (e * s.dst_esize != drb) { ok = false; break; }
                s.row_elems = e;
                for (size_t k = 0; k < s.srcs.size(); ++k) {
                    if (s.src_row[k]) {
                        if (s.ncols < 1 || e % s.ncols) { ok = false; break; }
                        s.src_rb[k] = 0;
                    } else {
                        s.src_rb[k] = e * s.src_esize[k];
                    }
                    need(s.srcs[k], s.src_rb[k]);
                }
                break;
            }
            case StepKind::GemmExact:
            case StepKind::GemmTc: {
                if (s.batch != 1 || s.M != R || s.a_col || s.N * s.dst_esize != drb ||
                    s.src_esize.size() != s.srcs.size()) {
                    ok = false;
                    break;
                }
                s.src_rb[0] = s.K * s.src_esize[0];
                need(s.srcs[0], s.src_rb[0]);
                need(s.srcs[1], 0);
                for (size_t k = 2; k < s.srcs.size(); ++k) {
                    s.src_rb[k] = s.src_row[k] ? 0 : s.N * s.src_esize[k];
                    need(s.srcs[k], s.src_rb[k]);
                }
                if (s.aux.size() == 3) {               // A_lo, A_hi split like A; B_lo stays whole
                    s.aux_rb[0] = s.K * 4;
                    s.aux_rb[2] = s.K * 4;
                    need(s.aux[0], s.aux_rb[0]);
                    need(s.aux[1], 0);
                    need(s.aux[2], s.aux_rb[2]);
                } else if (!s.aux.empty()) {
                    ok = false;
                }
                break;
            }
            default:
                ok = false;
        }
    }
    if (!ok) {
        for (auto& s : P.steps) {
            s.panel = false;
            s.dst_rb = 0;
            s.row_elems = 0;
            s.src_rb.assign(s.srcs.size(), 0);
            s.aux_rb.assign(s.aux.size(), 0);
        }
        analyse_column_streaming(P, R);
        return;
    }
    for (int k = 0; k < P.n_inputs; ++k) {
        auto it = rb.find({(int)BufRef::In, k});
        P.in_rb[k] = it == rb.end() ? 0 : it->second;
    }
    P.out_rb = P.out_bytes / R;
    P.stream_rows = R;
    // Panel boundaries fall on multiples of 256 rows: whole CTA-pair tiles
    // for a GEMM, 16-byte aligned offsets for the vectorised kernels.
    P.stream_align = 256;
    P.stream_ok = true;
}

}  // namespace bafe_cuda
