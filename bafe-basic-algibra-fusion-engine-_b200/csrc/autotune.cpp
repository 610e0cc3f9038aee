// autotune.cpp -- the B200 roofline cost model and device-timed autotuning.
//
// BAFE's optimizer prices graphs with a roofline model built from a
// bafe_hardware_model (cost.c:73-107) whose stock instances describe CPUs
// (cost.c:25-67), and its autotune loop logs (features, predicted cost,
// observed ms) records, refits a linear model of log(ms) by least squares
// and invalidates cached kernels (profiling.c).  With this backend the
// kernels run on a B200, so:
//
//   * bafe_cuda_hardware_model fills BAFE's hardware struct with the B200's
//     figures -- HBM and L2 streaming bandwidth, the f32 GEMM rate of the
//     precision in use and the rates of the other dtypes relative to it --
//     measured on the device by bafe_cuda_calibrate (nominal figures until
//     then);
//   * bafe_cuda_plan_predict_ms prices a lowered plan step by step with
//     that model (max(flops / rate, bytes / bandwidth) + launch latency);
//   * observed times are DEVICE times: CUDA events around the kernels of a
//     host call (bafe_cuda_plan_last_device_ms) or around device-resident
//     runs (bafe_cuda_time_device), never wall clock around PCIe copies;
//   * the profiling log, feature vector, refit and autotune configuration
//     restate profiling.c so that records and learned models are
//     interchangeable with BAFE's own; bafe_cuda_autotune_dispatch is the
//     working form of bafe_autotune_dispatch (profiling.c:364-410 only logs
//     nothing and returns 0; BAFE's Python layer does the timing).
#include "internal.h"

#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#define BAFE_API extern "C" __attribute__((visibility("default")))

namespace bafe_cuda {
namespace {

// ------------------------------------------------------------ calibration --

struct Calibration {
    bool done = false;
    double hbm_gbs = 0;            // streaming read+write bandwidth, > L2 working set
    double l2_gbs = 0;             // the same with an L2-resident working set
    double launch_us = 0;          // one small launch, back to back
    double tc3_tflops = 0;         // f32 GEMM, 3xTF32 tensor cores (4096^3)
    double tc1_tflops = 0;         // f32 GEMM, TF32 tensor cores (4096^3)
    double exact_tflops[6] = {0, 0, 0, 0, 0, 0};   // exact CUDA-core GEMM per dtype
};
Calibration g_cal[64];

// Nominal B200 figures used before calibration (dense, per GPU).
constexpr double kNominalHbmGbs = 7700.0;
constexpr double kNominalL2Gbs = 21000.0;
constexpr double kNominalTf32Tflops = 1100.0;
constexpr double kNominalLaunchUs = 4.0;
// exact CUDA-core GEMM (no FMA, chunked order): per dtype, nominal
constexpr double kNominalExact[6] = {40.0, 20.0, 20.0, 5.0, 40.0, 40.0};

// A bafe_graph assembled in C++ (the calibration workloads).
struct GraphMaker {
    bafe_graph* g;
    GraphMaker() : g(new bafe_graph()) { memset(g, 0, sizeof(bafe_graph)); }
    ~GraphMaker() { delete g; }
    int node(const char* op, std::initializer_list<int64_t> dims, int dtype) {
        const int id = g->n_nodes++;
        bafe_node& n = g->nodes[id];
        n.id = id;
        n.op_name = op;
        n.shape.rank = (int32_t)dims.size();
        int r = 0;
        for (int64_t d : dims) n.shape.dims[r++] = (int32_t)d;
        n.dtype = (bafe_dtype)dtype;
        n.layout = BAFE_LAYOUT_ROW_MAJOR;
        return id;
    }
    int input(const char* name, std::initializer_list<int64_t> dims, int dtype) {
        const int id = node("input", dims, dtype);
        bafe_node& n = g->nodes[id];
        n.is_input = true;
        snprintf(n.input_name, sizeof(n.input_name), "%s", name);
        snprintf(n.attrs.name, sizeof(n.attrs.name), "%s", name);
        g->inputs[g->n_inputs++] = id;
        return id;
    }
    int op(const char* name, std::initializer_list<int> ch, std::initializer_list<int64_t> dims, int dtype) {
        const int id = node(name, dims, dtype);
        bafe_node& n = g->nodes[id];
        for (int c : ch) n.children[n.n_children++] = c;
        return id;
    }
    void output(int id) { g->outputs[g->n_outputs++] = id; }
};

// Compiles the graph under the current options and times `iters` device
// runs on freshly allocated buffers (inputs filled from `fill`, cycled).
int time_graph(const bafe_graph* g, const std::vector<float>& fill, int iters, double& ms, std::string& err) {
    char ebuf[512];
    bafe_kernel_fn fn = bafe_cuda_jit_get_or_compile(g, ebuf, sizeof(ebuf));
    if (!fn) { err = ebuf; return 2; }
    std::lock_guard<std::recursive_mutex> lk(api_mutex());
    Plan* p = find_plan(plan_id_of(fn));
    if (!p) { err = "calibration plan vanished"; return 10; }
    std::vector<void*> bufs;
    int rc = 0;
    auto bytes_of = [&](int k) { return k < p->n_inputs ? p->in_bytes[k] : p->out_bytes; };
    for (int k = 0; k <= p->n_inputs && !rc; ++k) {
        void* d = nullptr;
        if (cudaMalloc(&d, (size_t)bytes_of(k)) != cudaSuccess) {
            cudaGetLastError();
            err = "cudaMalloc failed during calibration";
            rc = 6;
            break;
        }
        bufs.push_back(d);
        if (k < p->n_inputs) {
            // repeat the fill pattern over the buffer
            const size_t fb = fill.size() * sizeof(float);
            for (size_t off = 0; off < (size_t)bytes_of(k) && !rc; off += fb) {
                size_t nb = std::min(fb, (size_t)bytes_of(k) - off);
                if (cudaMemcpy(static_cast<char*>(d) + off, fill.data(), nb, cudaMemcpyHostToDevice) != cudaSuccess) {
                    cudaGetLastError();
                    err = "cudaMemcpy failed during calibration";
                    rc = 7;
                }
            }
        }
    }
    if (!rc) {
        rc = time_plan_device(*p, bufs.data(), (int)bufs.size(), nullptr, iters, ms);
        if (rc) { std::string m; get_error(m); err = m; }
    }
    for (void* d : bufs) cudaFree(d);
    return rc;
}

// ----------------------------------------------------------- profiling --
// Restatement of profiling.c's state and algorithms.

bafe_profiling_log g_log;
bafe_learned_cost_model g_model;
bafe_autotune_config g_config;
bafe_autotune_stats g_stats;
int g_since_refit = 0;
bool g_init = false;

bafe_autotune_config config_default() {
    bafe_autotune_config c;
    memset(&c, 0, sizeof(c));
    c.enabled = false;
    c.refit_threshold = 20;
    c.invalidation_drift = 0.25;
    c.warmup_calls = 2;
    c.timing_iters = 5;
    return c;
}

void ensure_init() {
    if (g_init) return;
    g_config = config_default();
    memset(&g_log, 0, sizeof(g_log));
    memset(&g_model, 0, sizeof(g_model));
    memset(&g_stats, 0, sizeof(g_stats));
    g_init = true;
}

size_t numel(const bafe_shape& s) {
    if (s.rank == 0) return 1;
    size_t n = 1;
    for (int i = 0; i < s.rank; ++i) {
        if (s.dims[i] < 0) return 0;
        n *= (size_t)s.dims[i];
    }
    return n;
}

size_t dtype_bytes(int d) {
    static const size_t b[6] = {4, 8, 4, 8, 2, 2};
    return d < 0 || d > 5 ? 4 : b[d];
}

// FLOPs of one node as BAFE's cost model counts them (cost.c:118-165),
// including its use of B's second-to-last dimension for N in a matmul, so
// that feature vectors match BAFE's exactly.
double node_flops(const char* op, const bafe_shape* in, int n_in, const bafe_shape& out) {
    auto is = [&](const char* s) { return strcmp(op, s) == 0; };
    if (is("matmul") && n_in == 2) {
        const double M = in[0].dims[in[0].rank - 2], K = in[0].dims[in[0].rank - 1];
        const double N = in[1].dims[in[1].rank - 2];
        int32_t batch = 1;
        for (int i = 0; i < in[0].rank - 2; ++i) batch *= in[0].dims[i];
        return 2.0 * M * N * K * (double)batch;
    }
    if (is("fused_matmul_relu") && n_in == 2) return node_flops("matmul", in, 2, out);
    if ((is("fused_matmul_bias") || is("fused_matmul_bias_relu")) && n_in == 3)
        return node_flops("matmul", in, 2, out) + (double)numel(out);
    const double n = (double)numel(out);
    if (is("add") || is("sub") || is("mul") || is("neg") || is("relu")) return n;
    if (is("sigmoid") || is("tanh")) return 4.0 * n;
    if (is("bias_add") || is("scale")) return n;
    if (is("reduce_sum") || is("reduce_max")) return n_in > 0 ? (double)numel(in[0]) : 0.0;
    if (is("fused_bias_relu")) return 2.0 * n;
    return 0.0;
}

// Bytes of one node (cost.c:168-177): every operand and the output at the
// node's element size.
double node_bytes(const bafe_shape* in, int n_in, const bafe_shape& out, int dtype) {
    const double es = (double)dtype_bytes(dtype);
    double r = 0.0;
    for (int i = 0; i < n_in; ++i) r += (double)numel(in[i]) * es;
    return r + (double)numel(out) * es;
}

bool is_fused(const char* op) { return op && strncmp(op, "fused_", 6) == 0; }

void extract_features(const bafe_graph* g, double* f) {
    for (int i = 0; i < BAFE_NUM_FEATURES; ++i) f[i] = 0.0;
    if (!g) return;
    int n_ops = 0, n_mm = 0, n_fused = 0, n_inter = 0;
    double flops = 0.0, bytes = 0.0;
    bool col = false;
    for (int i = 0; i < g->n_nodes; ++i) {
        const bafe_node& n = g->nodes[i];
        if (n.is_input || n.is_constant) continue;
        const char* op = n.op_name ? n.op_name : "";
        ++n_ops;
        if (strcmp(op, "matmul") == 0) ++n_mm;
        if (is_fused(op)) ++n_fused;
        if (n.layout == BAFE_LAYOUT_COL_MAJOR) col = true;
        if (!is_fused(op) && strcmp(op, "transpose") && strcmp(op, "reshape") && strcmp(op, "broadcast_to") &&
            strcmp(op, "layout_transform"))
            ++n_inter;
        bafe_shape ch[BAFE_MAX_CHILDREN];
        const int nc = n.n_children < BAFE_MAX_CHILDREN ? n.n_children : BAFE_MAX_CHILDREN;
        for (int j = 0; j < nc; ++j) {
            const int c = n.children[j];
            ch[j] = c >= 0 && c < g->n_nodes ? g->nodes[c].shape : bafe_shape{};
        }
        flops += node_flops(op, ch, nc, n.shape);
        bytes += node_bytes(ch, nc, n.shape, n.dtype);
    }
    f[0] = (double)g->n_inputs;
    f[1] = (double)n_ops;
    f[2] = (double)n_mm;
    f[3] = (double)n_fused;
    f[4] = std::log(flops + 1.0);
    f[5] = std::log(bytes + 1.0);
    f[6] = (double)n_inter;
    f[7] = col ? 1.0 : 0.0;
}

void log_add(const char* hash, const double* f, double predicted, double observed, int kernel_id) {
    bafe_profiling_record& r = g_log.records[g_log.head];
    memset(r.graph_hash, 0, sizeof(r.graph_hash));
    if (hash) strncpy(r.graph_hash, hash, 64);
    for (int i = 0; i < BAFE_NUM_FEATURES; ++i) r.features[i] = f ? f[i] : 0.0;
    r.predicted_cost = predicted;
    r.observed_ms = observed;
    r.kernel_id = kernel_id;
    g_log.head = (g_log.head + 1) % BAFE_PROFILING_LOG_SIZE;
    if (g_log.n < BAFE_PROFILING_LOG_SIZE) ++g_log.n;
    else g_log.wrapped = true;
    ++g_since_refit;
}

// Least squares fit of log(observed_ms) = bias + w . features over the log
// (records with observed_ms <= 0 skipped): normal equations X^T X p = X^T y
// solved by Gaussian elimination with partial pivoting; pivots below 1e-12
// leave their parameter at 0.  Same method and conventions as BAFE's refit
// (profiling.c:210-320), so both produce the same model from the same log.
int refit() {
    if (g_log.n < 5) return -1;
    constexpr int P = BAFE_NUM_FEATURES + 1;
    const int start = g_log.wrapped ? g_log.head : 0;
    double A[P][P + 1];
    memset(A, 0, sizeof(A));
    auto each = [&](auto&& fn) {
        for (int i = 0; i < g_log.n; ++i) {
            const bafe_profiling_record& r = g_log.records[(start + i) % BAFE_PROFILING_LOG_SIZE];
            if (r.observed_ms <= 0.0) continue;
            double x[P];
            x[0] = 1.0;
            for (int j = 0; j < BAFE_NUM_FEATURES; ++j) x[j + 1] = r.features[j];
            fn(x, std::log(r.observed_ms));
        }
    };
    each([&](const double* x, double y) {
        for (int a = 0; a < P; ++a) {
            for (int c = 0; c < P; ++c) A[a][c] += x[a] * x[c];
            A[a][P] += x[a] * y;
        }
    });
    for (int col = 0; col < P; ++col) {
        int best = col;
        for (int r = col + 1; r < P; ++r)
            if (std::fabs(A[r][col]) > std::fabs(A[best][col])) best = r;
        if (std::fabs(A[best][col]) < 1e-12) continue;
        if (best != col)
            for (int c = 0; c <= P; ++c) std::swap(A[col][c], A[best][c]);
        for (int r = col + 1; r < P; ++r) {
            const double f = A[r][col] / A[col][col];
            for (int c = col; c <= P; ++c) A[r][c] -= f * A[col][c];
        }
    }
    double w[P];
    for (int i = P - 1; i >= 0; --i) {
        double s = A[i][P];
        for (int j = i + 1; j < P; ++j) s -= A[i][j] * w[j];
        w[i] = std::fabs(A[i][i]) > 1e-12 ? s / A[i][i] : 0.0;
    }
    double mean = 0.0;
    int used = 0;
    each([&](const double*, double y) { mean += y; ++used; });
    if (used > 0) mean /= used;
    double ss_tot = 0.0, ss_res = 0.0;
    each([&](const double* x, double y) {
        double pred = 0.0;
        for (int j = 0; j < P; ++j) pred += w[j] * x[j];
        ss_tot += (y - mean) * (y - mean);
        ss_res += (y - pred) * (y - pred);
    });
    double r2 = ss_tot > 1e-12 ? 1.0 - ss_res / ss_tot : 0.0;
    if (r2 < 0.0) r2 = 0.0;
    g_model.bias = w[0];
    for (int j = 0; j < BAFE_NUM_FEATURES; ++j) g_model.weights[j] = w[j + 1];
    g_model.r_squared = r2;
    g_model.n_samples = used;
    g_model.valid = true;
    ++g_stats.total_refits;
    g_stats.last_refit_r_squared = r2;
    g_since_refit = 0;
    return 0;
}

double predict_log(const double* f) {
    if (!g_model.valid || !f) return 0.0;
    double p = g_model.bias;
    for (int j = 0; j < BAFE_NUM_FEATURES; ++j) p += g_model.weights[j] * f[j];
    return p;
}

// ------------------------------------------------------------ roofline --

struct Rates {
    double hbm_Bps, l2_Bps, launch_s, l2_bytes;
    double tc3, tc1;               // flop/s
    double exact[6];
};

Rates rates_for(int dev) {
    Rates r;
    const Calibration* c = dev >= 0 && dev < 64 && g_cal[dev].done ? &g_cal[dev] : nullptr;
    r.hbm_Bps = (c ? c->hbm_gbs : kNominalHbmGbs) * 1e9;
    r.l2_Bps = (c ? c->l2_gbs : kNominalL2Gbs) * 1e9;
    r.launch_s = (c ? c->launch_us : kNominalLaunchUs) * 1e-6;
    r.tc1 = (c ? c->tc1_tflops : kNominalTf32Tflops) * 1e12;
    r.tc3 = (c ? c->tc3_tflops : kNominalTf32Tflops / 3.0) * 1e12;
    for (int d = 0; d < 6; ++d) r.exact[d] = (c && c->exact_tflops[d] > 0 ? c->exact_tflops[d] : kNominalExact[d]) * 1e12;
    int l2 = 0;
    if (dev >= 0 && cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, dev) != cudaSuccess) {
        cudaGetLastError();
        l2 = 0;
    }
    r.l2_bytes = l2 > 0 ? (double)l2 : 126.0 * 1024 * 1024;
    return r;
}

double stream_time(const Rates& r, double bytes) {
    return bytes / (bytes <= r.l2_bytes ? r.l2_Bps : r.hbm_Bps);
}

double step_seconds(const Step& s, const Rates& r, int gemm_dtype) {
    switch (s.kind) {
        case StepKind::Ew: {
            double b = (double)s.n * s.dst_esize * (s.has_dst2 ? 2 : 1);
            for (size_t k = 0; k < s.srcs.size(); ++k)
                b += (double)(s.src_row[k] ? s.ncols : s.n) * s.src_esize[k];
            return stream_time(r, b);
        }
        case StepKind::GemmTc:
        case StepKind::GemmExact: {
            const double flops = 2.0 * (double)s.M * s.N * s.K * s.batch;
            double b = (double)s.M * s.N * s.dst_esize * s.batch;
            for (size_t k = 0; k < s.srcs.size() && k < s.src_esize.size(); ++k) {
                if (k == 0) b += (double)s.M * s.K * s.src_esize[k] * (s.a_bstride ? s.batch : 1);
                else if (k == 1) b += (double)s.K * s.N * s.src_esize[k] * (s.b_bstride ? s.batch : 1);
                else b += (double)(s.src_row[k] ? s.N : s.M * s.N) * s.src_esize[k];
            }
            if (s.kind == StepKind::GemmTc && s.tc_variant == 3 && !s.tc_convert) b += (double)(s.M * s.K + s.K * s.N) * 4.0;
            const double rate = s.kind == StepKind::GemmTc ? (s.tc_variant == 3 ? r.tc3 : r.tc1)
                                                           : r.exact[gemm_dtype >= 0 && gemm_dtype < 6 ? gemm_dtype : 0];
            return std::max(flops / rate, stream_time(r, b));
        }
        case StepKind::Transpose2d: return stream_time(r, 2.0 * (double)s.M * s.N * s.dst_esize);
        case StepKind::Gather: return stream_time(r, 2.0 * (double)s.n * s.dst_esize);
        case StepKind::Reduce: return stream_time(r, (double)s.M * s.N * (s.src_esize.empty() ? 4 : s.src_esize[0]));
        case StepKind::Zero: return stream_time(r, (double)s.dst_bytes);
    }
    return 0.0;
}

double plan_predict_seconds(const Plan& p, int dev) {
    const Rates r = rates_for(dev);
    double t = 0.0;
    for (const Step& s : p.steps) {
        // the exact kernel computes in the wider of the operand types; its
        // rate is keyed by the first operand's stored element size class
        int dt = BAFE_DTYPE_F32;
        if (s.kind == StepKind::GemmExact && !s.src_esize.empty()) {
            const int es = s.src_esize[0];
            dt = es == 8 ? BAFE_DTYPE_F64 : es == 2 ? BAFE_DTYPE_BF16 : BAFE_DTYPE_F32;
        }
        t += step_seconds(s, r, dt) + r.launch_s;
    }
    return t;
}

int current_device() {
    int dev = options().device;
    if (dev < 0 && cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    return dev;
}

}  // namespace
}  // namespace bafe_cuda

using namespace bafe_cuda;

// --------------------------------------------------------- hardware model --

BAFE_API int bafe_cuda_calibrate(int device, int what) {
    if (device < 0 || device >= 64) { set_error(4, "device ordinal out of range"); return 4; }
    int prev = -1;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) {
        cudaGetLastError();
        set_error(4, "cannot select CUDA device " + std::to_string(device));
        return 4;
    }
    Calibration c = g_cal[device];
    std::string err;
    int rc = 0;
    // Deterministic, non-constant operand values (power draw of the tensor
    // cores depends on the data).
    std::vector<float> fill(1 << 20);
    uint32_t st = 12345u;
    for (float& v : fill) {
        st = st * 1664525u + 1013904223u;
        v = (float)((int32_t)(st >> 8) - (1 << 23)) / (float)(1 << 23);
    }
    const std::string prec = options().gemm_precision;
    if (what & 1) {
        // streaming bandwidth: out = relu(x), 2^27 f32 (512 MiB in + out)
        GraphMaker big;
        int x = big.input("x", {1 << 27}, BAFE_DTYPE_F32);
        big.output(big.op("relu", {x}, {1 << 27}, BAFE_DTYPE_F32));
        double ms = 0;
        if (!(rc = time_graph(big.g, fill, 10, ms, err))) c.hbm_gbs = 2.0 * 4.0 * (1 << 27) / (ms * 1e-3) / 1e9;
        // L2-resident: 2^22 f32 (16 MiB in + out)
        GraphMaker mid;
        x = mid.input("x", {1 << 22}, BAFE_DTYPE_F32);
        mid.output(mid.op("relu", {x}, {1 << 22}, BAFE_DTYPE_F32));
        if (!rc && !(rc = time_graph(mid.g, fill, 50, ms, err))) c.l2_gbs = 2.0 * 4.0 * (1 << 22) / (ms * 1e-3) / 1e9;
        // launch latency: 1024 elements
        GraphMaker tiny;
        x = tiny.input("x", {1024}, BAFE_DTYPE_F32);
        tiny.output(tiny.op("relu", {x}, {1024}, BAFE_DTYPE_F32));
        if (!rc && !(rc = time_graph(tiny.g, fill, 100, ms, err))) c.launch_us = ms * 1e3;
    }
    auto gemm_rate = [&](int n, int dtype, const char* precision, int iters, double& tflops) {
        GraphMaker m;
        int a = m.input("A", {n, n}, dtype), b = m.input("B", {n, n}, dtype);
        m.output(m.op("matmul", {a, b}, {n, n}, dtype));
        options().gemm_precision = precision;
        double ms = 0;
        int r = time_graph(m.g, fill, iters, ms, err);
        options().gemm_precision = prec;
        if (!r) tflops = 2.0 * n * (double)n * n / (ms * 1e-3) / 1e12;
        return r;
    };
    if (!rc && (what & 2)) {
        rc = gemm_rate(4096, BAFE_DTYPE_F32, "3xtf32", 10, c.tc3_tflops);
        if (!rc) rc = gemm_rate(4096, BAFE_DTYPE_F32, "tf32", 10, c.tc1_tflops);
        if (!rc) rc = gemm_rate(2048, BAFE_DTYPE_F32, "exact", 3, c.exact_tflops[BAFE_DTYPE_F32]);
    }
    if (!rc && (what & 4)) {
        const int others[] = {BAFE_DTYPE_F64, BAFE_DTYPE_I32, BAFE_DTYPE_I64, BAFE_DTYPE_F16, BAFE_DTYPE_BF16};
        for (int d : others)
            if (!rc) rc = gemm_rate(1024, d, "exact", 3, c.exact_tflops[d]);
    }
    if (prev >= 0) cudaSetDevice(prev);
    if (rc) {
        set_error(rc, "calibration failed: " + err);
        return rc;
    }
    c.done = true;
    g_cal[device] = c;
    return 0;
}

BAFE_API int bafe_cuda_hardware_model(int device, bafe_hardware_model* h) {
    if (!h) return -1;
    if (device < 0) device = current_device();
    int sms = 148, clock_khz = 1965000, smem = 233472, l2 = 126 << 20;
    if (device >= 0) {
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
        cudaDeviceGetAttribute(&clock_khz, cudaDevAttrClockRate, device);
        cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerMultiprocessor, device);
        cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, device);
        cudaGetLastError();
    }
    const Rates r = rates_for(device);
    const std::string& prec = options().gemm_precision;
    const double f32 = prec == "tf32" ? r.tc1 : prec == "exact" ? r.exact[BAFE_DTYPE_F32] : r.tc3;
    memset(h, 0, sizeof(*h));
    h->peak_gflops = f32 / 1e9;
    h->clock_ghz = clock_khz / 1e6;
    h->simd_width = 32;                                   // threads of a warp
    // On-chip capacity a kernel's working set spreads over: every SM's
    // shared memory / L1, then the L2; there is no third level, so "L3" is
    // the L2 again and anything larger streams from HBM.
    h->l1_cache_size = (int)std::min<long long>((long long)smem * sms, 0x7FFFFFFF);
    h->l2_cache_size = l2;
    h->l3_cache_size = l2;
    h->l1_bandwidth_gbs = (double)sms * 128.0 * h->clock_ghz;   // 128 B / clock / SM
    h->l2_bandwidth_gbs = r.l2_Bps / 1e9;
    h->l3_bandwidth_gbs = r.l2_Bps / 1e9;
    h->dram_bandwidth_gbs = r.hbm_Bps / 1e9;
    // dtype rates relative to the f32 GEMM path (BAFE scales flops by these)
    h->f32_flop_rate = 1.0;
    h->f64_flop_rate = r.exact[BAFE_DTYPE_F64] / f32;
    h->f16_flop_rate = r.exact[BAFE_DTYPE_F16] / f32;
    h->bf16_flop_rate = r.exact[BAFE_DTYPE_BF16] / f32;
    h->i32_flop_rate = r.exact[BAFE_DTYPE_I32] / f32;
    h->i64_flop_rate = r.exact[BAFE_DTYPE_I64] / f32;
    return g_cal[device >= 0 && device < 64 ? device : 0].done ? 1 : 0;
}

BAFE_API double bafe_cuda_plan_predict_ms(int plan) {
    std::lock_guard<std::recursive_mutex> lk(api_mutex());
    Plan* p = find_plan(plan);
    if (!p) return -1.0;
    return plan_predict_seconds(*p, current_device()) * 1e3;
}

// ---------------------------------------------------------- device timing --

BAFE_API double bafe_cuda_plan_last_device_ms(int plan) {
    std::lock_guard<std::recursive_mutex> lk(api_mutex());
    Plan* p = find_plan(plan);
    return p ? p->last_device_ms : -1.0;
}

BAFE_API int bafe_cuda_time_device(int plan, void* const* ptrs, int n_ptrs, void* stream, int iters, double* ms) {
    std::lock_guard<std::recursive_mutex> lk(api_mutex());
    Plan* p = find_plan(plan);
    if (!p) { set_error(10, "unknown plan " + std::to_string(plan)); return 10; }
    double t = -1.0;
    int rc = time_plan_device(*p, ptrs, n_ptrs, stream, iters, t);
    if (ms) *ms = t;
    return rc;
}

// -------------------------------------------------------------- profiling --

BAFE_API void bafe_cuda_profiling_init(void) { ensure_init(); }

BAFE_API void bafe_cuda_profiling_reset(void) {
    memset(&g_log, 0, sizeof(g_log));
    memset(&g_model, 0, sizeof(g_model));
    memset(&g_stats, 0, sizeof(g_stats));
    g_since_refit = 0;
    if (!g_init) g_config = config_default();
    g_init = true;
}

BAFE_API void bafe_cuda_profiling_extract_features(const bafe_graph* g, double* features) {
    ensure_init();
    if (features) extract_features(g, features);
}

BAFE_API void bafe_cuda_profiling_add(const char* graph_hash, const double* features, double predicted_cost,
                                      double observed_ms, int kernel_id) {
    ensure_init();
    log_add(graph_hash, features, predicted_cost, observed_ms, kernel_id);
}

BAFE_API const bafe_profiling_log* bafe_cuda_profiling_get_log(void) {
    ensure_init();
    return &g_log;
}

BAFE_API int bafe_cuda_profiling_dump_jsonl(const char* path) {
    ensure_init();
    if (!path) return -1;
    FILE* f = fopen(path, "w");
    if (!f) return -1;
    const int start = g_log.wrapped ? g_log.head : 0;
    for (int i = 0; i < g_log.n; ++i) {
        const bafe_profiling_record& r = g_log.records[(start + i) % BAFE_PROFILING_LOG_SIZE];
        fprintf(f, "{\"hash\":\"%.16s\",\"features\":[", r.graph_hash);
        for (int j = 0; j < BAFE_NUM_FEATURES; ++j) fprintf(f, "%s%.6f", j ? "," : "", r.features[j]);
        fprintf(f, "],\"predicted\":%.6f,\"observed_ms\":%.6f,\"kernel_id\":%d}\n", r.predicted_cost, r.observed_ms,
                r.kernel_id);
    }
    fclose(f);
    return g_log.n;
}

BAFE_API int bafe_cuda_profiling_refit(void) {
    ensure_init();
    return refit();
}

BAFE_API const bafe_learned_cost_model* bafe_cuda_profiling_get_model(void) {
    ensure_init();
    return &g_model;
}

BAFE_API double bafe_cuda_profiling_predict_log(const double* features) {
    ensure_init();
    return predict_log(features);
}

BAFE_API double bafe_cuda_profiling_predict_ms(const double* features) {
    ensure_init();
    return std::exp(predict_log(features));
}

BAFE_API bafe_autotune_config bafe_cuda_autotune_config_default(void) { return config_default(); }

BAFE_API void bafe_cuda_autotune_configure(const bafe_autotune_config* cfg) {
    ensure_init();
    if (cfg) g_config = *cfg;
}

BAFE_API bafe_autotune_config bafe_cuda_autotune_get_config(void) {
    ensure_init();
    return g_config;
}

BAFE_API bafe_autotune_stats bafe_cuda_autotune_get_stats(void) {
    ensure_init();
    g_stats.log_size = g_log.n;
    return g_stats;
}

BAFE_API double bafe_cuda_autotune_dispatch(bafe_kernel_fn fn, void** args, int n_args, const bafe_graph* graph,
                                            const char* graph_hash, double predicted_cost) {
    ensure_init();
    if (!fn || !args || n_args <= 0) return -1.0;
    std::lock_guard<std::recursive_mutex> lk(api_mutex());
    const int pid = plan_id_of(fn);
    Plan* p = find_plan(pid);
    if (!p) { set_error(10, "autotune dispatch: not a live bafe_cuda kernel"); return -1.0; }
    if (n_args != p->n_inputs + 1) {
        set_error(8, "autotune dispatch: plan takes " + std::to_string(p->n_inputs + 1) + " pointers");
        return -1.0;
    }
    ++g_stats.total_calls;
    if (g_stats.total_calls <= g_config.warmup_calls) {
        // warm-up: run (the caller wants the result) but do not log
        return run_plan_host(*p, args, n_args) ? -1.0 : 0.0;
    }
    const int iters = g_config.timing_iters > 0 ? g_config.timing_iters : 1;
    double total = 0.0;
    for (int i = 0; i < iters; ++i) {
        if (run_plan_host(*p, args, n_args)) return -1.0;
        total += p->last_device_ms;
    }
    const double observed = total / iters;
    double f[BAFE_NUM_FEATURES];
    extract_features(graph, f);
    const double predicted = predicted_cost > 0.0 ? predicted_cost : plan_predict_seconds(*p, current_device()) * 1e3;
    log_add(graph_hash ? graph_hash : p->graph_hash.c_str(), f, predicted, observed, pid);
    if (g_config.refit_threshold > 0 && g_since_refit >= g_config.refit_threshold && refit() == 0) {
        // the refitted model disagrees with what was just measured: drop
        // the cached plans so the next compile re-plans with it
        const double pred_ms = std::exp(predict_log(f));
        if (observed > 0.0 && std::fabs(pred_ms - observed) / observed > g_config.invalidation_drift) {
            ++g_stats.total_invalidations;
            drop_memory_cache();
        }
    }
    return observed;
}
