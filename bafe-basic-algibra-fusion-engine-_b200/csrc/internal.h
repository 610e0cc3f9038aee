// internal.h -- shared declarations of libbafe_cuda.so's host runtime.
//
// Pipeline (one call of bafe_cuda_jit_get_or_compile):
//   parse_graph   bafe_graph (BAFE's POD struct) -> Graph (validated, typed)
//   lower_graph   Graph -> Plan: fusion into launch steps + generated CUDA
//                 source for all of the plan's kernels (one module)
//   compile       NVRTC -> sm_100a cubin, cached on disk by source hash
//   run           driver-API module load (lazily, per device), launches
#pragma once

#include "bafe_cuda.h"

#include <cstdint>
#include <mutex>
#include <string>
#include <vector>

namespace bafe_cuda {

// ---------------------------------------------------------------- graph --

enum class Op {
    Input, Constant, MatMul, Add, Sub, Mul, BiasAdd, Relu, Neg, Sigmoid, Tanh,
    Transpose, ReduceSum, ReduceMax, Reshape, BroadcastTo, LayoutTransform,
    FusedMatmulRelu, FusedMatmulBias, FusedMatmulBiasRelu, FusedBiasRelu,
    Unknown
};

struct Shape {
    int rank = 0;
    int64_t d[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int64_t numel() const {
        int64_t n = 1;
        for (int i = 0; i < rank; ++i) n *= d[i];
        return n;
    }
    bool same(const Shape& o) const {
        if (rank != o.rank) return false;
        for (int i = 0; i < rank; ++i) if (d[i] != o.d[i]) return false;
        return true;
    }
    std::string str() const;
};

struct Node {
    int id = -1;
    Op op = Op::Unknown;
    std::string opname;
    std::vector<int> ch;
    Shape shape;
    int dtype = BAFE_DTYPE_F32;
    int layout = BAFE_LAYOUT_ROW_MAJOR;
    int input_index = -1;          // position in g->inputs (kernel parameter order)
    std::string name;
    std::vector<int> perm, axes, tshape;
    bool keepdims = false;
};

struct Graph {
    std::vector<Node> nodes;
    std::vector<int> inputs;       // node ids in parameter order
    int root = -1;
};

int parse_graph(const bafe_graph* g, Graph& out, std::string& err);
int hash_graph(const bafe_graph* g, char* out, size_t out_size);

// Byte size of one stored element of a BAFE dtype.
int dtype_size(int dtype);
// Compute type the emitter uses for a node of this dtype (F16/BF16 -> F32).
int compute_dtype(int dtype);
const char* dtype_ctype(int dtype);   // device C type of the STORAGE (u16 for halves)

// -------------------------------------------------------------- options --

struct Options {
    std::string gemm_precision = "auto";   // auto | 3xtf32 | tf32 | exact
    int device = -1;                        // -1: current device
    bool tc_pair = true;                    // tensor-core GEMM on CTA pairs (cta_group::2)
    int host_panels = -1;                   // host calls: -1 auto, 0/1 off, n: n row panels
    int tc_convert = -1;                    // 3xTF32 residuals inside the kernel: 1 yes, 0 no, -1 auto (small GEMMs)
    int kslice_free_sms = 0;                // K-sliced runs: SMs every slice but the last leaves to other streams
    bool host_graphs = true;                // small host calls replay as one CUDA graph
};
Options& options();

// ----------------------------------------------------------------- plan --

struct BufRef {
    enum Kind { In, Tmp, Out } kind = Tmp;
    int idx = 0;
};

enum class StepKind { Ew, GemmExact, GemmTc, Transpose2d, Gather, Reduce, Zero };

struct Step {
    StepKind kind = StepKind::Ew;
    std::string kernel;            // entry point (extern "C") in the plan's module
    std::string kernel_vec;        // Ew: vectorised entry point ("" if none); GemmTc: split-tail fixup
    BufRef dst;
    BufRef dst2;                   // Ew: a second output, same element count (has_dst2)
    bool has_dst2 = false;
    std::vector<BufRef> srcs;      // operands in kernel argument order
    int64_t dst_bytes = 0;
    // Ew / Zero
    int64_t n = 0, ncols = 1;
    std::vector<int> src_esize;    // Ew: stored element size of each operand
    std::vector<bool> src_row;     // Ew: operand indexed by column (row vector)
    int dst_esize = 4;
    // GEMM
    int64_t M = 0, N = 0, K = 0, batch = 1;
    int64_t a_bstride = 0, b_bstride = 0, o_bstride = 0;
    int a_col = 0, b_col = 0;
    int n_epi = 0;                 // epilogue operands are srcs[2..2+n_epi)
    bool direct = false;           // fused-form summation order (one chunk)
    int exact_tm = 4;              // GemmExact: outputs per thread and axis (tile 16 * exact_tm)
    int tc_variant = 0;            // GemmTc: 1 = tf32, 3 = 3xtf32
    bool tc_pair = false;          // GemmTc: CTA-pair kernel (256x256 tiles)
    int tc_elem = 0;               // GemmTc operands: 0 = f32 (tf32 MMAs), 1 = bf16 (kind::f16)
    bool tc_convert = false;       // GemmTc 3xTF32: residuals made in shared memory (no aux buffers)
    std::vector<BufRef> aux;       // GemmTc 3xtf32: A_lo, B_lo, B_hi (the operand parts the pre-passes write)
    // Row streaming of host calls (analyse_row_streaming): the step runs
    // once per row panel of the output (panel) or once per call; buffers
    // with a nonzero byte count per row are offset to the panel's first row.
    bool panel = false;
    int64_t row_elems = 0;         // Ew: elements per output row
    int64_t dst_rb = 0;
    std::vector<int64_t> src_rb, aux_rb;
    // Transpose2d (output M x N), Gather, Reduce
    int64_t gdims[8] = {0}, gstride[8] = {0};
    int grank = 0;
    int axis = 0;
    std::string describe;
};

struct DeviceState;   // per-device runtime state of a plan (runtime.cpp)

struct Plan {
    int id = -1;
    std::string graph_hash;
    std::string key;               // graph hash + lowering options
    int n_inputs = 0;
    std::vector<int> in_dtypes;
    std::vector<int64_t> in_bytes;
    int out_dtype = BAFE_DTYPE_F32;
    int64_t out_bytes = 0;
    std::vector<int64_t> tmp_bytes;
    std::vector<Step> steps;
    // Row streaming: host calls may copy the row-split inputs, run the
    // panel steps and copy the output back panel by panel on three streams.
    bool stream_ok = false;
    int64_t stream_rows = 0;       // rows of the output (leading dimension)
    int64_t stream_align = 1;      // panel boundaries are multiples of this
    std::vector<int64_t> in_rb;    // bytes per output row of each input (0: whole)
    // A plan that is one rank-2 transpose of input 0 into the output streams
    // by output rows too, but each panel's input is a band of x's COLUMNS
    // (a strided copy); stream_ok stays false (bafe_cuda_plan_row_split
    // reports row splits only).
    bool stream_cols = false;
    int64_t out_rb = 0;
    std::string source;            // generated CUDA for every step's kernel
    std::string source_hash;       // key of the cubin
    std::string cubin;             // compiled image (kept for lazy per-device loads)
    std::string describe;
    std::vector<DeviceState*> dev; // indexed by device ordinal
    double last_device_ms = -1.0;  // kernel time of the last host call (CUDA events)
};

// Lower a parsed graph into steps + generated source.  Host-only: needs no
// GPU.  Returns 0 or a nonzero code with a message in err.
int lower_graph(const Graph& g, const Options& opt, Plan& plan, std::string& err);
// Decides which steps and buffers split by output row (fills the row
// streaming fields of the plan and its steps).
void analyse_row_streaming(Plan& plan, const Shape& out_shape);

// Embedded kernel headers (generated at build time from csrc/kernels/*.cuh).
struct EmbeddedHeader { const char* name; const char* text; };
extern const EmbeddedHeader kEmbeddedHeaders[];
extern const int kNumEmbeddedHeaders;

// NVRTC compile with on-disk cache.  Returns 0, or nonzero with err set.
int compile_cubin(const std::string& source, const std::string& source_hash,
                  std::string& cubin, bool& from_cache, std::string& err);
std::string cache_dir();
void set_cache_dir(const std::string& d);

// SHA-256 of a byte string, lowercase hex.
std::string sha256_hex(const void* data, size_t len);

// Runtime (runtime.cpp).
int run_plan_device(Plan& p, void* const* ptrs, int n_ptrs, void* stream);
// The plan (tf32 pre-passes + one CTA-pair GEMM) over K slices
// [k_bounds[j], k_bounds[j+1]); slice j's launches wait for ready[j] (a
// cudaEvent_t, or null).  plan_k_slice_align: the multiple of K slice
// bounds must be, 0 if the plan cannot be sliced.
int run_plan_device_ksliced(Plan& p, void* const* ptrs, int n_ptrs, void* stream, int n_slices,
                            const int64_t* k_bounds, void* const* ready);
int plan_k_slice_align(const Plan& p);
// run_plan_device with step_events[2i] / [2i+1] (cudaEvent_t) recorded on the
// stream before / after step i's launches.
int run_plan_device_timed(Plan& p, void* const* ptrs, int n_ptrs, void* stream, void* const* step_events,
                          int n_events);
// resident: per input, nonzero = ptrs[k] is already a device buffer (or null: none);
// ready: cudaEvent_t the kernels wait for before reading them (or null)
int run_plan_host(Plan& p, void* const* ptrs, int n_ptrs, const unsigned char* resident = nullptr,
                  void* ready = nullptr);
// Synchronises the current device and reports a kernel-raised error word.
int synchronize_current_device();
void release_plan_device_state(Plan& p);

// Plan registry (api.cpp), for the autotuning entry points.
std::recursive_mutex& api_mutex();
Plan* find_plan(int id);
int plan_id_of(bafe_kernel_fn fn);
void drop_memory_cache();

// Device timing of a plan on device buffers: mean ms of `iters` runs after
// one untimed run (autotune.cpp).
int time_plan_device(Plan& p, void* const* ptrs, int n_ptrs, void* stream, int iters, double& ms);

// Error slot shared by every entry point.
void set_error(int code, const std::string& msg);
int  get_error(std::string& msg);
void clear_error();

extern int64_t g_launch_count;

}  // namespace bafe_cuda
