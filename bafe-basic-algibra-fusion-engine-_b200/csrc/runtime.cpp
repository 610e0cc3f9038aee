// runtime.cpp -- compile (NVRTC, on-disk cubin cache), load (CUDA driver
// API), run (launch steps on device buffers; host calls stage through
// device buffers the plan owns).
//
// The CUDA runtime is linked statically and loads the driver lazily, so the
// library loads -- and plans compile -- on a machine without a GPU; the
// first launch then fails with a recorded error instead.
#include "internal.h"
#include "tc_launch.h"

#include <cuda.h>
#include <cuda_runtime.h>
#include <nvrtc.h>

#include <algorithm>
#include <cerrno>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <mutex>
#include <sstream>
#include <sys/stat.h>
#include <unistd.h>

namespace bafe_cuda {

int64_t g_launch_count = 0;

// --------------------------------------------------------------- errors --

namespace {
int g_err_code = 0;
std::string g_err_msg;
}  // namespace

void set_error(int code, const std::string& msg) {
    g_err_code = code;
    g_err_msg = msg;
}
int get_error(std::string& msg) {
    msg = g_err_msg;
    return g_err_code;
}
void clear_error() {
    g_err_code = 0;
    g_err_msg.clear();
}

// ----------------------------------------------------------- cache dir --

namespace {
std::string g_cache_dir;
bool g_cache_dir_set = false;

void mkdirs(const std::string& path) {
    std::string cur;
    for (size_t i = 0; i < path.size(); ++i) {
        cur += path[i];
        if (path[i] == '/' && cur.size() > 1) mkdir(cur.c_str(), 0755);
    }
    mkdir(path.c_str(), 0755);
}
}  // namespace

// $BAFE_CACHE_DIR, else $HOME/.bafecache, else ./.bafecache (jit.c:173-189).
std::string cache_dir() {
    if (g_cache_dir_set) return g_cache_dir;
    const char* env = getenv("BAFE_CACHE_DIR");
    if (env && *env) g_cache_dir = env;
    else if (const char* home = getenv("HOME")) g_cache_dir = std::string(home) + "/.bafecache";
    else g_cache_dir = ".bafecache";
    g_cache_dir_set = true;
    return g_cache_dir;
}
void set_cache_dir(const std::string& d) {
    g_cache_dir = d;
    g_cache_dir_set = true;
}

// --------------------------------------------------------------- NVRTC --

namespace {
std::string headers_digest() {
    static std::string d;
    if (d.empty()) {
        std::string all;
        for (int i = 0; i < kNumEmbeddedHeaders; ++i) {
            all += kEmbeddedHeaders[i].name;
            all += '\0';
            all += kEmbeddedHeaders[i].text;
            all += '\0';
        }
        d = sha256_hex(all.data(), all.size());
    }
    return d;
}

const char* kNvrtcOpts[] = {
    "--gpu-architecture=sm_100a",
    "-std=c++17",
    // No contraction anywhere: the reference's C rounds every op.
    "--fmad=false",
    "-lineinfo",
    "-DBAFE_NVRTC=1",
};
}  // namespace

int compile_cubin(const std::string& source, const std::string& source_hash, std::string& cubin,
                  bool& from_cache, std::string& err) {
    from_cache = false;
    int major = 0, minor = 0;
    nvrtcVersion(&major, &minor);
    std::string keysrc = source_hash + "|" + headers_digest() + "|nvrtc" + std::to_string(major) + "." +
                         std::to_string(minor);
    for (const char* o : kNvrtcOpts) keysrc += std::string("|") + o;
    const std::string key = sha256_hex(keysrc.data(), keysrc.size());
    const std::string dir = cache_dir() + "/cuda";
    const std::string path = dir + "/" + key + ".cubin";
    {
        std::ifstream f(path, std::ios::binary);
        if (f) {
            std::ostringstream ss;
            ss << f.rdbuf();
            cubin = ss.str();
            if (cubin.size() > 16 && memcmp(cubin.data(), "\x7f" "ELF", 4) == 0) {
                from_cache = true;
                return 0;
            }
            cubin.clear();   // corrupt entry: recompile and overwrite
        }
    }
    std::vector<const char*> names, texts;
    for (int i = 0; i < kNumEmbeddedHeaders; ++i) {
        names.push_back(kEmbeddedHeaders[i].name);
        texts.push_back(kEmbeddedHeaders[i].text);
    }
    nvrtcProgram prog;
    nvrtcResult r = nvrtcCreateProgram(&prog, source.c_str(), "bafe_plan.cu", (int)names.size(), texts.data(),
                                       names.data());
    if (r != NVRTC_SUCCESS) {
        err = std::string("nvrtcCreateProgram: ") + nvrtcGetErrorString(r);
        return 3;
    }
    std::vector<const char*> opts(std::begin(kNvrtcOpts), std::end(kNvrtcOpts));
    if (getenv("BAFE_PTXAS_VERBOSE")) opts.push_back("--ptxas-options=-v");
    r = nvrtcCompileProgram(prog, (int)opts.size(), opts.data());
    size_t log_size = 0;
    nvrtcGetProgramLogSize(prog, &log_size);
    std::string log(log_size, '\0');
    if (log_size) nvrtcGetProgramLog(prog, &log[0]);
    if (getenv("BAFE_PTXAS_VERBOSE") && log_size > 1) fprintf(stderr, "[bafe_cuda] nvrtc log:\n%s\n", log.c_str());
    if (r != NVRTC_SUCCESS) {
        err = std::string("compile failed: ") + nvrtcGetErrorString(r) + "\n" + log.substr(0, 4000);
        nvrtcDestroyProgram(&prog);
        return 3;
    }
    size_t n = 0;
    nvrtcGetCUBINSize(prog, &n);
    cubin.assign(n, '\0');
    nvrtcGetCUBIN(prog, &cubin[0]);
    nvrtcDestroyProgram(&prog);
    // Atomic publish: concurrent ranks may compile the same key.
    mkdirs(dir);
    const std::string tmp = path + ".tmp." + std::to_string((long long)getpid());
    {
        std::ofstream f(tmp, std::ios::binary);
        f.write(cubin.data(), (std::streamsize)cubin.size());
    }
    if (rename(tmp.c_str(), path.c_str()) != 0) unlink(tmp.c_str());
    return 0;
}

// -------------------------------------------------------- driver table --

namespace {
struct Driver {
    bool ok = false;
    std::string why;
    decltype(&cuModuleLoadData) moduleLoadData = nullptr;
    decltype(&cuModuleUnload) moduleUnload = nullptr;
    decltype(&cuModuleGetFunction) moduleGetFunction = nullptr;
    decltype(&cuFuncSetAttribute) funcSetAttribute = nullptr;
    decltype(&cuLaunchKernelEx) launchKernelEx = nullptr;
    decltype(&cuTensorMapEncodeTiled) tensorMapEncodeTiled = nullptr;
    decltype(&cuGetErrorString) getErrorString = nullptr;
};

Driver& driver() {
    static Driver d;
    static bool init = false;
    if (init) return d;
    init = true;
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0) {
        d.why = std::string("no CUDA device available (") + cudaGetErrorString(e) + ")";
        cudaGetLastError();
        return d;
    }
    auto get = [&](const char* name, void** fn) {
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint(name, fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !*fn) {
            d.why = std::string("driver entry point missing: ") + name;
            return false;
        }
        return true;
    };
    if (!get("cuModuleLoadData", (void**)&d.moduleLoadData)) return d;
    if (!get("cuModuleUnload", (void**)&d.moduleUnload)) return d;
    if (!get("cuModuleGetFunction", (void**)&d.moduleGetFunction)) return d;
    if (!get("cuFuncSetAttribute", (void**)&d.funcSetAttribute)) return d;
    if (!get("cuLaunchKernelEx", (void**)&d.launchKernelEx)) return d;
    if (!get("cuTensorMapEncodeTiled", (void**)&d.tensorMapEncodeTiled)) return d;
    if (!get("cuGetErrorString", (void**)&d.getErrorString)) return d;
    d.ok = true;
    return d;
}

std::string cu_err(CUresult r) {
    const char* s = nullptr;
    if (driver().getErrorString) driver().getErrorString(r, &s);
    return s ? s : ("CUresult " + std::to_string((int)r));
}

int sm_count(int dev) {
    static int cache[64] = {0};
    if (dev < 0 || dev >= 64) return 148;
    if (!cache[dev]) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = v > 0 ? v : 148;
    }
    return cache[dev];
}
}  // namespace

// Driver calls used by the tensor-core launcher (tc_launch.cpp).
int tc_encode_tensor_map(void* map, int elem, int rank, void* gaddr, const uint64_t* dims,
                         const uint64_t* strides_bytes, const uint32_t* box, int swizzle, std::string& err) {
    Driver& d = driver();
    if (!d.ok) { err = d.why; return 4; }
    cuuint64_t gd[5], gs[4];
    cuuint32_t bx[5], es[5];
    for (int i = 0; i < rank; ++i) { gd[i] = dims[i]; bx[i] = box[i]; es[i] = 1; }
    for (int i = 0; i < rank - 1; ++i) gs[i] = strides_bytes[i];
    CUresult r = d.tensorMapEncodeTiled(
        reinterpret_cast<CUtensorMap*>(map),
        elem == 1 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                  : (elem == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8),
        (cuuint32_t)rank, gaddr, gd, gs, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
        swizzle == 2 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                     : (swizzle == 1 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE),
        CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) { err = "cuTensorMapEncodeTiled: " + cu_err(r); return 4; }
    return 0;
}

// ------------------------------------------------------ device state --

struct DeviceState {
    int device = -1;
    CUmodule module = nullptr;
    std::vector<CUfunction> fn, fn_vec;
    std::vector<void*> tmp;
    std::vector<void*> in_stage;        // inputs' device copies: in_block + in_off[k]
    void* in_block = nullptr;           // one allocation for all of them
    std::vector<int64_t> in_off;        // 256-byte aligned offsets in in_block
    int64_t in_block_bytes = 0;
    void* out_stage = nullptr;
    cudaStream_t stream = nullptr;      // host calls: kernels
    cudaStream_t h2d = nullptr;         // host calls: input copies (row streaming)
    cudaStream_t d2h = nullptr;         // host calls: output copies (row streaming)
    std::vector<cudaEvent_t> events;    // row streaming: per-panel hand-offs
    std::vector<cudaEvent_t> tev;       // host calls: timing events around the kernels
    // Prepared tensor-core launches (tensor maps + argument block) per step,
    // reused while the buffers and panel rows are the same: encoding four
    // tensor maps per call is host work that small GEMMs would wait for.
    struct TcCached {
        bool valid = false;
        const void* key[15] = {};   // a, b, a_lo, b_lo, out, error word, 8 epilogue operands, workspace
        int64_t rows = 0;
        TcLaunch L;
    };
    std::vector<TcCached> tc_cache;
    // Partial tiles of split tensor-core GEMMs (grown on demand; every
    // split step of the plan runs on `stream`, one after another).
    void* tc_ws = nullptr;
    size_t tc_ws_bytes = 0;
    // Wave-alignment counter of the tensor-core GEMMs (zeroed before each
    // launch that uses it; the plan's GEMMs run one after another).
    unsigned* tc_ctr = nullptr;
    // Pinned host buffer of small host calls (kPackedCallBytes at most).
    void* host_stage = nullptr;
    size_t host_stage_bytes = 0;
    // Pinned copy of the device error word, read on `stream` at the end of
    // a host call (a synchronous read would add a blocking copy per call).
    unsigned* err_host = nullptr;
    // Packed small host calls replayed as one CUDA graph (the copy in, the
    // plan's launches, the copies out, the timing events): every pointer in
    // them is this state's own, so the second such call captures them and
    // later calls launch the graph.
    cudaGraphExec_t graph_exec = nullptr;
    int64_t graph_kernels = 0;          // kernels per replay (the launch counter)
    int packed_calls = 0;
    bool graph_failed = false;          // capture failed once: stay eager
};

// Host calls moving at most this many bytes in total copy through one
// pinned buffer: a copy from pageable memory is a synchronous staged copy
// with a fixed cost that dominates small calls; from pinned memory the
// copies queue behind one another and run asynchronously.
constexpr int64_t kPackedCallBytes = int64_t(1) << 20;
// ... and move all their inputs in one copy, pinned ones included, up to
// this many input bytes.
constexpr int64_t kPackPinnedBytes = int64_t(128) << 10;

// Timing events (pairs: before / after kernels) of a host call.
static int ensure_timing_events(DeviceState* ds, size_t n) {
    while (ds->tev.size() < n) {
        cudaEvent_t ev = nullptr;
        if (cudaEventCreate(&ev) != cudaSuccess) {
            cudaGetLastError();
            set_error(6, "cudaEventCreate failed");
            return 6;
        }
        ds->tev.push_back(ev);
    }
    return 0;
}

// Sum of the kernel intervals recorded in tev[0..2*pairs) (synchronised).
static double timed_ms(DeviceState* ds, size_t pairs) {
    double total = 0.0;
    for (size_t i = 0; i < pairs; ++i) {
        float ms = 0.0f;
        if (cudaEventElapsedTime(&ms, ds->tev[2 * i], ds->tev[2 * i + 1]) != cudaSuccess) {
            cudaGetLastError();
            return -1.0;
        }
        total += ms;
    }
    return total;
}

// One device word per GPU that kernels with bounded waits report a timeout
// into (0 = ok).  Allocated on first use of the device.
namespace {
unsigned* g_err_word[64] = {nullptr};
}
unsigned* device_error_word(int dev) {
    if (dev < 0 || dev >= 64) return nullptr;
    if (!g_err_word[dev]) {
        void* p = nullptr;
        if (cudaMalloc(&p, 4) != cudaSuccess) { cudaGetLastError(); return nullptr; }
        cudaMemset(p, 0, 4);
        g_err_word[dev] = static_cast<unsigned*>(p);
    }
    return g_err_word[dev];
}

namespace {

int ensure_device_state(Plan& p, int dev, DeviceState*& out) {
    Driver& d = driver();
    if (!d.ok) { set_error(4, d.why); return 4; }
    if ((int)p.dev.size() <= dev) p.dev.resize(dev + 1, nullptr);
    if (p.dev[dev]) { out = p.dev[dev]; return 0; }
    DeviceState* s = new DeviceState();
    s->device = dev;
    cudaFree(nullptr);   // make the device's primary context current
    CUresult r = d.moduleLoadData(&s->module, p.cubin.data());
    if (r != CUDA_SUCCESS) {
        set_error(5, "cuModuleLoadData: " + cu_err(r));
        delete s;
        return 5;
    }
    for (auto& st : p.steps) {
        CUfunction f = nullptr, fv = nullptr;
        if (!st.kernel.empty()) {
            r = d.moduleGetFunction(&f, s->module, st.kernel.c_str());
            if (r != CUDA_SUCCESS) {
                set_error(5, "cuModuleGetFunction(" + st.kernel + "): " + cu_err(r));
                d.moduleUnload(s->module);
                delete s;
                return 5;
            }
            if (st.kind == StepKind::GemmTc) {
                r = d.funcSetAttribute(f, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                                       tc_smem_bytes(st.tc_variant, st.tc_pair));
                if (r != CUDA_SUCCESS) {
                    set_error(5, "cuFuncSetAttribute(smem): " + cu_err(r));
                    d.moduleUnload(s->module);
                    delete s;
                    return 5;
                }
            }
        }
        if (!st.kernel_vec.empty()) d.moduleGetFunction(&fv, s->module, st.kernel_vec.c_str());
        s->fn.push_back(f);
        s->fn_vec.push_back(fv);
    }
    p.dev[dev] = s;
    out = s;
    return 0;
}

int alloc(void** ptr, int64_t bytes) {
    *ptr = nullptr;
    if (bytes <= 0) return 0;
    cudaError_t e = cudaMalloc(ptr, (size_t)bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error(6, "cudaMalloc(" + std::to_string((long long)bytes) + "): " + cudaGetErrorString(e));
        return 6;
    }
    return 0;
}

int launch(CUfunction f, unsigned gx, unsigned gy, unsigned gz, unsigned bx, unsigned by, unsigned bz,
           unsigned smem, cudaStream_t stream, void** params) {
    CUlaunchConfig cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDimX = gx; cfg.gridDimY = gy; cfg.gridDimZ = gz;
    cfg.blockDimX = bx; cfg.blockDimY = by; cfg.blockDimZ = bz;
    cfg.sharedMemBytes = smem;
    cfg.hStream = (CUstream)stream;
    CUresult r = driver().launchKernelEx(&cfg, f, params, nullptr);
    if (r != CUDA_SUCCESS) {
        set_error(7, "kernel launch failed: " + cu_err(r));
        return 7;
    }
    ++g_launch_count;
    return 0;
}

unsigned grid_for(int64_t units, int dev) {
    int64_t g = (units + 255) / 256;
    int64_t cap = (int64_t)sm_count(dev) * 8;
    if (g > cap) g = cap;
    if (g < 1) g = 1;
    return (unsigned)g;
}

// Host mirrors of the kernels' by-value argument structs (layouts must
// match csrc/kernels/*.cuh).
struct GemmArgsHost {
    const void* a; const void* b; void* out;
    int64_t M, N, K, batch;
    int64_t a_bstride, b_bstride, o_bstride;
    int32_t a_col, b_col;
    const void* ep[8];
    int64_t z0, y0;
};
static_assert(sizeof(GemmArgsHost) == 168, "GemmArgs layout");
struct GatherArgsHost {
    int64_t numel;
    int32_t rank;
    int64_t dims[8];
    int64_t stride[8];
};
static_assert(sizeof(GatherArgsHost) == 144, "GatherArgs layout");

int ensure_tmps(Plan& p, DeviceState* ds) {
    if (ds->tmp.size() != p.tmp_bytes.size()) {
        ds->tmp.assign(p.tmp_bytes.size(), nullptr);
        for (size_t t = 0; t < p.tmp_bytes.size(); ++t)
            if (int rc = alloc(&ds->tmp[t], p.tmp_bytes[t])) return rc;
    }
    return 0;
}

// Which steps one pass of run_steps launches: all of them over the whole
// problem, only the once-per-call steps, or the per-panel steps over output
// rows [r0, r0 + rows).
// KPrep / KSlice: a plan of tf32 pre-passes and one CTA-pair GEMM run over
// K slices (run_plan_device_ksliced): KPrep runs A's residual pre-pass over
// all of A; KSlice runs B's split pre-pass over rows [k0, k1) of B and the
// GEMM over K range [k0, k1), continuing (first false) and leaving (last
// false) its sums in the output.
struct Pass {
    enum Kind { All, Once, Panel, KPrep, KSlice } kind = All;
    int64_t r0 = 0, rows = 0;
    int64_t k0 = 0, k1 = 0;
    bool first = true, last = true;
    const cudaEvent_t* step_events = nullptr;   // All: recorded before / after each step (2 per step)
};

bool same_buf(const BufRef& a, const BufRef& b) { return a.kind == b.kind && a.idx == b.idx; }

// Role of step si in a K-sliced plan: 0 the GEMM (last step), 1 A's split
// pre-pass (writes aux[0] = A_lo and aux[2] = A_hi), 2 B's residual pre-pass
// (writes aux[1] = B_lo), -1 anything else (the plan cannot be sliced).
int k_slice_role(const Plan& p, size_t si) {
    const Step& G = p.steps.back();
    const Step& s = p.steps[si];
    if (si + 1 == p.steps.size()) return 0;
    if (s.kind != StepKind::Ew || G.aux.size() < 3 || s.srcs.size() != 1) return -1;
    if (s.has_dst2 && same_buf(s.dst, G.aux[0]) && same_buf(s.dst2, G.aux[2]) && same_buf(s.srcs[0], G.srcs[0]))
        return 1;
    if (!s.has_dst2 && same_buf(s.dst, G.aux[1]) && same_buf(s.srcs[0], G.srcs[1])) return 2;
    return -1;
}

int run_steps(Plan& p, DeviceState* ds, int dev, void* const* ptrs, cudaStream_t stream, const Pass& pass) {
    auto ptr_of = [&](const BufRef& b) -> void* {
        switch (b.kind) {
            case BufRef::In: return ptrs[b.idx];
            case BufRef::Tmp: return ds->tmp[b.idx];
            default: return ptrs[p.n_inputs];
        }
    };
    const bool cut = pass.kind == Pass::Panel;
    // a buffer of a panel step, moved to the panel's first row
    auto at_row = [&](void* base, int64_t row_bytes) -> void* {
        return cut && row_bytes ? static_cast<void*>(static_cast<char*>(base) + pass.r0 * row_bytes) : base;
    };
    const bool ksl = pass.kind == Pass::KPrep || pass.kind == Pass::KSlice;
    for (size_t si = 0; si < p.steps.size(); ++si) {
        Step& s = p.steps[si];
        if (pass.kind == Pass::Once && s.panel) continue;
        if (pass.kind == Pass::Panel && !s.panel) continue;
        // K slices: A's split once (KPrep); B's residual over the slice's
        // rows of B and the GEMM over its K range (KSlice)
        const int role = ksl ? k_slice_role(p, si) : -1;
        if (ksl && (pass.kind == Pass::KPrep) != (role == 1)) continue;
        if (ksl && role == 2) {
            const int64_t off = pass.k0 * p.steps.back().N;            // B row-major: rows are contiguous
            const int64_t cnt = (pass.k1 - pass.k0) * p.steps.back().N;
            if (cnt == 0) continue;
            char* bsrc = static_cast<char*>(ptr_of(s.srcs[0])) + off * s.src_esize[0];
            char* lo = static_cast<char*>(ptr_of(s.dst)) + off * 4;
            const bool vec = ds->fn_vec[si] != nullptr && ((uintptr_t)bsrc | (uintptr_t)lo) % 16 == 0;
            uint64_t args[4] = {(uint64_t)(uintptr_t)bsrc, (uint64_t)(uintptr_t)lo, (uint64_t)cnt, (uint64_t)s.ncols};
            void* params[] = {args};
            if (int rc = launch(vec ? ds->fn_vec[si] : ds->fn[si], grid_for(vec ? cnt / 4 : cnt, dev), 1, 1, 256, 1, 1, 0,
                                stream, params))
                return rc;
            continue;
        }
        void* dst = at_row(ptr_of(s.dst), s.dst_rb);
        const int64_t n_run = cut ? pass.rows * s.row_elems : s.n;
        if (pass.step_events) cudaEventRecord(pass.step_events[2 * si], stream);
        const int64_t m_run = cut ? pass.rows : s.M;
        switch (s.kind) {
            case StepKind::Zero: {
                if (s.dst_bytes > 0) {
                    cudaError_t e = cudaMemsetAsync(dst, 0, (size_t)s.dst_bytes, stream);
                    if (e != cudaSuccess) { cudaGetLastError(); set_error(7, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e)); return 7; }
                }
                break;
            }
            case StepKind::Ew: {
                if (n_run == 0) break;
                std::vector<uint64_t> args;
                bool vec = ds->fn_vec[si] != nullptr;
                for (size_t k = 0; k < s.srcs.size(); ++k) {
                    void* q = at_row(ptr_of(s.srcs[k]), s.src_rb.empty() ? 0 : s.src_rb[k]);
                    args.push_back((uint64_t)(uintptr_t)q);
                    uintptr_t need = s.src_esize[k] == 2 ? 8 : 16;
                    if ((uintptr_t)q % need) vec = false;
                    if (s.src_row[k] && (s.ncols % 4)) vec = false;
                }
                if ((uintptr_t)dst % (s.dst_esize == 2 ? 8 : 16)) vec = false;
                args.push_back((uint64_t)(uintptr_t)dst);
                args.push_back((uint64_t)n_run);
                args.push_back((uint64_t)s.ncols);
                if (s.has_dst2) {                            // second output: same rows as dst
                    void* d2 = at_row(ptr_of(s.dst2), s.dst_rb);
                    if ((uintptr_t)d2 % 16) vec = false;
                    args.push_back((uint64_t)(uintptr_t)d2);
                }
                void* params[] = {args.data()};
                int64_t units = vec ? n_run / 4 : n_run;
                if (int rc = launch(vec ? ds->fn_vec[si] : ds->fn[si], grid_for(units, dev), 1, 1, 256, 1, 1, 0,
                                    stream, params))
                    return rc;
                break;
            }
            case StepKind::GemmExact: {
                if (m_run == 0 || s.N == 0 || s.batch == 0) break;
                GemmArgsHost g;
                memset(&g, 0, sizeof(g));
                g.a = at_row(ptr_of(s.srcs[0]), s.src_rb.empty() ? 0 : s.src_rb[0]);
                g.b = ptr_of(s.srcs[1]);
                g.out = dst;
                g.M = m_run; g.N = s.N; g.K = s.K; g.batch = s.batch;
                g.a_bstride = s.a_bstride; g.b_bstride = s.b_bstride; g.o_bstride = s.o_bstride;
                g.a_col = s.a_col; g.b_col = s.b_col;
                for (int k = 0; k < s.n_epi; ++k)
                    g.ep[k] = at_row(ptr_of(s.srcs[2 + k]), s.src_rb.empty() ? 0 : s.src_rb[2 + k]);
                void* params[] = {&g};
                // grid (N tiles, M tiles, batch) of 16 * exact_tm wide tiles;
                // y and z stop at 65535, so larger problems launch in blocks
                // of 65535 (z0 / y0 offsets)
                const int64_t tile = 16 * s.exact_tm;
                const int64_t kMaxYZ = 65535, m_tiles = (m_run + tile - 1) / tile, nx = (s.N + tile - 1) / tile;
                if (nx > 0x7fffffff) { set_error(8, "GEMM grid too large"); return 8; }
                for (int64_t z0 = 0; z0 < s.batch; z0 += kMaxYZ)
                    for (int64_t y0 = 0; y0 < m_tiles; y0 += kMaxYZ) {
                        g.z0 = z0;
                        g.y0 = y0;
                        const int64_t nz = std::min(kMaxYZ, s.batch - z0), ny = std::min(kMaxYZ, m_tiles - y0);
                        if (int rc = launch(ds->fn[si], (unsigned)nx, (unsigned)ny, (unsigned)nz, 256, 1, 1, 0,
                                            stream, params))
                            return rc;
                    }
                break;
            }
            case StepKind::GemmTc: {
                std::vector<const void*> ep;
                for (int k = 0; k < s.n_epi; ++k)
                    ep.push_back(at_row(ptr_of(s.srcs[2 + k]), s.src_rb.empty() ? 0 : s.src_rb[2 + k]));
                unsigned* err_word = device_error_word(dev);
                if (!err_word) { set_error(6, "cannot allocate the device error word"); return 6; }
                std::string err;
                const void* a_lo = s.aux.size() > 0 ? at_row(ptr_of(s.aux[0]), s.aux_rb.empty() ? 0 : s.aux_rb[0]) : nullptr;
                const void* b_lo = s.aux.size() > 1 ? ptr_of(s.aux[1]) : nullptr;
                // 3xTF32 reads A's round-to-nearest hi part (aux[2], written by
                // the split pre-pass, row-split like A) and B's raw values
                const void* a = s.aux.size() > 2 ? at_row(ptr_of(s.aux[2]), s.aux_rb.size() > 2 ? s.aux_rb[2] : 0)
                                                 : at_row(ptr_of(s.srcs[0]), s.src_rb.empty() ? 0 : s.src_rb[0]);
                const void* b = ptr_of(s.srcs[1]);
                if (ds->tc_cache.size() != p.steps.size()) ds->tc_cache.assign(p.steps.size(), DeviceState::TcCached());
                DeviceState::TcCached& cached = ds->tc_cache[si];
                Step panel;                                  // the step over this call's rows
                if (cut) {
                    panel = s;
                    panel.M = m_run;
                }
                const Step& run = cut ? panel : s;
                // workspace for the partials of a split tail (none if it cannot be had)
                const size_t ws_need = ds->fn_vec[si] ? tc_split_of(run, sm_count(dev)).ws_bytes : 0;
                if (ws_need > ds->tc_ws_bytes) {
                    void* w = nullptr;
                    if (cudaMalloc(&w, ws_need) == cudaSuccess) {
                        if (ds->tc_ws) {
                            cudaStreamSynchronize(stream);   // earlier launches may still read the old one
                            cudaFree(ds->tc_ws);
                        }
                        ds->tc_ws = w;
                        ds->tc_ws_bytes = ws_need;
                    } else {
                        cudaGetLastError();
                    }
                }
                if (!ds->tc_ctr) {
                    void* c = nullptr;
                    if (cudaMalloc(&c, sizeof(unsigned)) == cudaSuccess) ds->tc_ctr = static_cast<unsigned*>(c);
                    else cudaGetLastError();                    // no alignment then
                }
                const void* key[15] = {a, b, a_lo, b_lo, dst, err_word};
                for (int k = 0; k < s.n_epi && k < 8; ++k) key[6 + k] = ep[k];
                key[14] = ds->tc_ws;
                TcLaunch sliced;                             // K slice: no split tail, not cached
                if (pass.kind == Pass::KSlice) {
                    if (int rc = tc_prepare(run, a, b, a_lo, b_lo, dst, ep, sm_count(dev), err_word, nullptr, 0,
                                            ds->tc_ctr, sliced, err)) {
                        set_error(rc, err);
                        return rc;
                    }
                    tc_set_k_slice(sliced, pass.k0, pass.k1, s.K, !pass.first, !pass.last, s.tc_elem == 1);
                    // every slice but the last may leave SMs to the streams that
                    // bring the next slabs in (a kernel queued there cannot start
                    // on an SM this persistent kernel fills)
                    const int free_pairs = (options().kslice_free_sms + 1) / 2;
                    const int pairs = sm_count(dev) / 2;
                    if (!pass.last && free_pairs > 0 && sliced.cluster == 2 && (int)sliced.grid / 2 > pairs - free_pairs)
                        sliced.grid = (unsigned)(2 * std::max(1, pairs - free_pairs));
                }
                bool hit = pass.kind == Pass::KSlice || (cached.valid && cached.rows == m_run);
                for (int k = 0; hit && k < 15; ++k) hit = cached.key[k] == key[k];
                if (!hit) {
                    int rc = tc_prepare(run, a, b, a_lo, b_lo, dst, ep, sm_count(dev), err_word,
                                        ds->fn_vec[si] ? ds->tc_ws : nullptr, ds->tc_ws_bytes, ds->tc_ctr, cached.L, err);
                    if (rc) {
                        cached.valid = false;
                        set_error(rc, err);
                        return rc;
                    }
                    for (int k = 0; k < 15; ++k) cached.key[k] = key[k];
                    cached.rows = m_run;
                    cached.valid = true;
                }
                TcLaunch& L = pass.kind == Pass::KSlice ? sliced : cached.L;
                if (L.wave_sync) {
                    cudaError_t e = cudaMemsetAsync(ds->tc_ctr, 0, sizeof(unsigned), stream);
                    if (e != cudaSuccess) { cudaGetLastError(); set_error(7, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e)); return 7; }
                }
                void* params[] = {L.args};
                CUlaunchConfig cfg;
                memset(&cfg, 0, sizeof(cfg));
                cfg.gridDimX = L.grid; cfg.gridDimY = 1; cfg.gridDimZ = 1;
                cfg.blockDimX = L.block; cfg.blockDimY = 1; cfg.blockDimZ = 1;
                cfg.sharedMemBytes = L.smem;
                cfg.hStream = (CUstream)stream;
                CUlaunchAttribute attr;
                memset(&attr, 0, sizeof(attr));
                if (L.cluster > 1) {
                    attr.id = CU_LAUNCH_ATTRIBUTE_CLUSTER_DIMENSION;
                    attr.value.clusterDim.x = L.cluster;
                    attr.value.clusterDim.y = 1;
                    attr.value.clusterDim.z = 1;
                    cfg.attrs = &attr;
                    cfg.numAttrs = 1;
                }
                CUresult r = driver().launchKernelEx(&cfg, ds->fn[si], params, nullptr);
                if (r != CUDA_SUCCESS) { set_error(7, "tensor-core GEMM launch failed: " + cu_err(r)); return 7; }
                ++g_launch_count;
                if (L.fix_grid) {                            // split tail tiles: sum the partials, epilogue
                    if (int rc = launch(ds->fn_vec[si], L.fix_grid, 1, 1, 256, 1, 1, 0, stream, params)) return rc;
                }
                break;
            }
            case StepKind::Transpose2d: {
                // a panel (column-streamed host call) is output rows
                // [r0, r0 + rows): x moved r0 columns (src_rb = one element),
                // out moved r0 rows (dst_rb), x's row length stays s.M
                if (m_run == 0 || s.N == 0 || s.batch < 1) break;
                const char* x0 = (const char*)at_row(ptr_of(s.srcs[0]), s.src_rb.empty() ? 0 : s.src_rb[0]);
                char* d0 = (char*)dst;
                const int64_t Nn = s.N, ldx = s.M, es = s.dst_esize;
                const bool vec = ds->fn_vec[si] && m_run % 4 == 0 && Nn % 4 == 0 && ldx % 4 == 0 &&
                                 ((uintptr_t)x0 | (uintptr_t)d0) % 16 == 0;
                // grid (N tiles, M tiles, batch); y and z stop at 65535.
                // Batch items go 65535 to a launch (base pointers moved by
                // whole items, which keeps the 16-byte alignment above).  If
                // M alone needs more than 65535 tiles, each item launches on
                // its own in blocks of rows: x moves by columns, out by rows,
                // ldx stays.
                const int64_t kMaxYZ = 65535, tile = vec ? 64 : 32;
                const int64_t m_tiles = (m_run + tile - 1) / tile;
                if ((Nn + tile - 1) / tile > 0x7fffffff) { set_error(8, "transpose grid too large"); return 8; }
                const int64_t rows_per = m_tiles > kMaxYZ ? kMaxYZ * tile : m_run;
                const int64_t items_per = m_tiles > kMaxYZ ? 1 : kMaxYZ;
                for (int64_t b0 = 0; b0 < s.batch; b0 += items_per)
                    for (int64_t r0 = 0; r0 < m_run; r0 += rows_per) {
                        const void* x = x0 + (b0 * ldx * Nn + r0) * es;
                        void* o = d0 + (b0 * m_run + r0) * Nn * es;
                        int64_t M = std::min(rows_per, m_run - r0);
                        const unsigned nb = (unsigned)std::min(items_per, s.batch - b0);
                        void* params[] = {&x, &o, &M, (void*)&Nn, (void*)&ldx};
                        const int rc = vec ? launch(ds->fn_vec[si], (unsigned)((Nn + 63) / 64), (unsigned)((M + 63) / 64),
                                                    nb, 256, 1, 1, 0, stream, params)
                                           : launch(ds->fn[si], (unsigned)((Nn + 31) / 32), (unsigned)((M + 31) / 32),
                                                    nb, 32, 8, 1, 0, stream, params);
                        if (rc) return rc;
                    }
                break;
            }
            case StepKind::Gather: {
                if (s.n == 0) break;
                const void* x = ptr_of(s.srcs[0]);
                GatherArgsHost g;
                memset(&g, 0, sizeof(g));
                g.numel = s.n;
                g.rank = s.grank;
                for (int d = 0; d < s.grank; ++d) { g.dims[d] = s.gdims[d]; g.stride[d] = s.gstride[d]; }
                void* params[] = {&x, &dst, &g};
                if (ds->fn_vec[si] && ((uintptr_t)x | (uintptr_t)dst) % 16 == 0) {
                    if (int rc = launch(ds->fn_vec[si], grid_for(s.n / 4, dev), 1, 1, 256, 1, 1, 0, stream, params))
                        return rc;
                    break;
                }
                if (int rc = launch(ds->fn[si], grid_for(s.n, dev), 1, 1, 256, 1, 1, 0, stream, params)) return rc;
                break;
            }
            case StepKind::Reduce: {
                const void* x = ptr_of(s.srcs[0]);
                int64_t M = s.M, Nn = s.N;
                int axis = s.axis;
                int64_t outs = axis == 0 ? s.N : s.M;
                if (outs == 0) break;
                void* params[] = {&x, &dst, &M, &Nn, &axis};
                if (int rc = launch(ds->fn[si], (unsigned)((outs + 255) / 256), 1, 1, 256, 1, 1, 0, stream, params))
                    return rc;
                break;
            }
        }
        if (pass.step_events) cudaEventRecord(pass.step_events[2 * si + 1], stream);
    }
    return 0;
}

}  // namespace

int run_plan_device_ksliced(Plan& p, void* const* ptrs, int n_ptrs, void* stream_v, int n_slices,
                            const int64_t* k_bounds, void* const* ready) {
    if (n_ptrs != p.n_inputs + 1) {
        set_error(8, "plan takes " + std::to_string(p.n_inputs + 1) + " pointers, got " + std::to_string(n_ptrs));
        return 8;
    }
    const int64_t align = p.steps.empty() ? 0 : tc_k_slice_align(p.steps.back());
    if (!align) {
        set_error(8, "K slices need a plan whose last step is a CTA-pair tensor-core GEMM with an fp32 output, "
                     "unbatched, B row-major");
        return 8;
    }
    for (size_t si = 0; si + 1 < p.steps.size(); ++si)
        if (k_slice_role(p, si) < 0) {
            set_error(8, "K slices: the plan has steps other than the GEMM's tf32 pre-passes");
            return 8;
        }
    const int64_t K = p.steps.back().K;
    if (n_slices < 1 || !k_bounds || k_bounds[0] != 0 || k_bounds[n_slices] != K) {
        set_error(8, "K slices: bounds must run from 0 to K = " + std::to_string(K));
        return 8;
    }
    for (int j = 0; j < n_slices; ++j)
        if (k_bounds[j + 1] <= k_bounds[j] || (j + 1 < n_slices && k_bounds[j + 1] % align)) {
            set_error(8, "K slices: bounds must increase and be multiples of " + std::to_string(align));
            return 8;
        }
    int dev = 0;
    cudaError_t ce = cudaGetDevice(&dev);
    if (ce != cudaSuccess) {
        cudaGetLastError();
        set_error(4, std::string("no CUDA device available (") + cudaGetErrorString(ce) + ")");
        return 4;
    }
    DeviceState* ds = nullptr;
    if (int rc = ensure_device_state(p, dev, ds)) return rc;
    if (int rc = ensure_tmps(p, ds)) return rc;
    cudaStream_t st = (cudaStream_t)stream_v;
    Pass prep;
    prep.kind = Pass::KPrep;
    if (int rc = run_steps(p, ds, dev, ptrs, st, prep)) return rc;
    for (int j = 0; j < n_slices; ++j) {
        if (ready && ready[j]) {
            cudaError_t e = cudaStreamWaitEvent(st, (cudaEvent_t)ready[j], 0);
            if (e != cudaSuccess) { cudaGetLastError(); set_error(7, std::string("cudaStreamWaitEvent: ") + cudaGetErrorString(e)); return 7; }
        }
        Pass sl;
        sl.kind = Pass::KSlice;
        sl.k0 = k_bounds[j];
        sl.k1 = k_bounds[j + 1];
        sl.first = j == 0;
        sl.last = j + 1 == n_slices;
        if (int rc = run_steps(p, ds, dev, ptrs, st, sl)) return rc;
    }
    return 0;
}

int run_plan_device_timed(Plan& p, void* const* ptrs, int n_ptrs, void* stream_v, void* const* step_events,
                          int n_events) {
    if (n_ptrs != p.n_inputs + 1) {
        set_error(8, "plan takes " + std::to_string(p.n_inputs + 1) + " pointers, got " + std::to_string(n_ptrs));
        return 8;
    }
    if (!step_events || n_events != 2 * (int)p.steps.size()) {
        set_error(8, "timed run: the plan has " + std::to_string(p.steps.size()) + " steps, so it takes " +
                         std::to_string(2 * p.steps.size()) + " events");
        return 8;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        set_error(4, "no CUDA device available");
        return 4;
    }
    DeviceState* ds = nullptr;
    if (int rc = ensure_device_state(p, dev, ds)) return rc;
    if (int rc = ensure_tmps(p, ds)) return rc;
    Pass pass;
    pass.step_events = reinterpret_cast<const cudaEvent_t*>(step_events);
    return run_steps(p, ds, dev, ptrs, (cudaStream_t)stream_v, pass);
}

int plan_k_slice_align(const Plan& p) {
    if (p.steps.empty()) return 0;
    for (size_t si = 0; si + 1 < p.steps.size(); ++si)
        if (k_slice_role(p, si) < 0) return 0;
    return tc_k_slice_align(p.steps.back());
}

int run_plan_device(Plan& p, void* const* ptrs, int n_ptrs, void* stream_v) {
    if (n_ptrs != p.n_inputs + 1) {
        set_error(8, "plan takes " + std::to_string(p.n_inputs + 1) + " pointers, got " + std::to_string(n_ptrs));
        return 8;
    }
    int dev = 0;
    cudaError_t ce = cudaGetDevice(&dev);
    if (ce != cudaSuccess) {
        cudaGetLastError();
        set_error(4, std::string("no CUDA device available (") + cudaGetErrorString(ce) + ")");
        return 4;
    }
    DeviceState* ds = nullptr;
    if (int rc = ensure_device_state(p, dev, ds)) return rc;
    if (int rc = ensure_tmps(p, ds)) return rc;
    return run_steps(p, ds, dev, ptrs, (cudaStream_t)stream_v, Pass());
}

// A kernel whose bounded wait expired wrote a nonzero code into the
// device's error word: report it (the output is not valid) and reset it.
// The caller has synchronised the work in question.
// A nonzero error word read back from device `dev`: clear it and report.
static int report_error_word(int dev, unsigned code) {
    if (!code) return 0;
    cudaMemset(g_err_word[dev], 0, 4);
    set_error(13, "tensor-core GEMM timed out waiting on a pipeline barrier (role code " + std::to_string(code) +
                      "); the output is invalid");
    return 13;
}

int check_device_error_word(int dev) {
    if (dev < 0 || dev >= 64 || !g_err_word[dev]) return 0;
    unsigned code = 0;
    if (cudaMemcpy(&code, g_err_word[dev], 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return report_error_word(dev, code);
}

int synchronize_current_device() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        set_error(4, "no CUDA device available");
        return 4;
    }
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error(9, std::string("device error: ") + cudaGetErrorString(e));
        return 9;
    }
    return check_device_error_word(dev);
}

namespace {

// Number of row panels a host call of plan p is split into (1 = not split).
int host_panel_count(const Plan& p) {
    if (!p.stream_ok && !p.stream_cols) return 1;
    const int want = options().host_panels;
    if (want == 0 || want == 1) return 1;
    const int64_t R = p.stream_rows, align = p.stream_align;
    const int64_t most = R / align;   // every panel but the last has >= align rows
    if (most < 2) return 1;
    int n = want;
    if (want < 0) {
        // Auto: split when the row-split traffic is large enough for the
        // copy / compute overlap to pay for the extra launches; one panel
        // per 96 MiB, 8 to 32 (the last panel's kernels and output copy are
        // the part that does not overlap: 16384^3 fused GEMM 66.9 ms with 8
        // panels, 63.5 with 32).
        int64_t per_row = p.out_rb;
        for (int64_t b : p.in_rb) per_row += b;
        const int64_t bytes = R * per_row;
        if (bytes < (int64_t(64) << 20)) return 1;
        const int64_t want_n = bytes / (int64_t(96) << 20);
        n = (int)(want_n < 8 ? 8 : want_n > 32 ? 32 : want_n);
    }
    return (int)(n < most ? n : most);
}

int sync_stream(cudaStream_t st) {
    cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error(9, std::string("device error: ") + cudaGetErrorString(e));
        return 9;
    }
    return 0;
}

int copy_async(void* dst, const void* src, int64_t bytes, cudaStream_t st, const char* what) {
    if (bytes <= 0) return 0;
    cudaError_t e = cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyDefault, st);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error(7, std::string(what) + ": " + cudaGetErrorString(e));
        return 7;
    }
    return 0;
}

// Row-streamed host call.  h2d stream: whole inputs, then each panel's rows
// of the split inputs; compute stream: the once-per-call steps after the
// whole inputs, then each panel's steps after its rows arrived; d2h stream:
// each panel's output rows after its steps.  All copies of one direction
// are issued before the other's, so with pageable host memory (whose copies
// the driver makes synchronous) the input copies still overlap the kernels.
int run_plan_host_streamed(Plan& p, DeviceState* ds, void* const* ptrs, int panels, const unsigned char* resident,
                           void* ready) {
    const int64_t R = p.stream_rows, align = p.stream_align;
    // Panel boundaries (multiples of align): the first and the last panel
    // are at most align rows each when there is room -- the kernels start
    // after a short first copy and the last output copy is short -- and the
    // rows between are split evenly into the remaining panels, large enough
    // to keep the kernels efficient.
    std::vector<std::pair<int64_t, int64_t>> bounds;   // (first row, rows)
    {
        int64_t lo = 0, hi = R;
        const bool ends = panels >= 4 && R >= (int64_t)(panels + 2) * align;
        if (ends) {
            bounds.push_back({0, align});
            lo = align;
            hi = (R - 1) / align * align;                // the last panel starts on a boundary too
        }
        const int mid = ends ? panels - 2 : panels;
        int64_t per = (hi - lo + mid - 1) / mid;
        per = (per + align - 1) / align * align;
        for (int64_t r = lo; r < hi; r += per) bounds.push_back({r, hi - r < per ? hi - r : per});
        if (ends) bounds.push_back({hi, R - hi});
        panels = (int)bounds.size();
    }
    for (cudaStream_t* st : {&ds->h2d, &ds->d2h}) {
        if (!*st && cudaStreamCreateWithFlags(st, cudaStreamNonBlocking) != cudaSuccess) {
            cudaGetLastError();
            set_error(6, "cudaStreamCreate failed");
            return 6;
        }
    }
    const size_t n_events = 2 * (size_t)panels + 1;
    while (ds->events.size() < n_events) {
        cudaEvent_t ev = nullptr;
        if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) {
            cudaGetLastError();
            set_error(6, "cudaEventCreate failed");
            return 6;
        }
        ds->events.push_back(ev);
    }
    if (int rc = ensure_timing_events(ds, 2 * (size_t)panels + 2)) return rc;
    cudaEvent_t whole = ds->events[0];
    auto in_done = [&](int i) { return ds->events[1 + 2 * i]; };
    auto run_done = [&](int i) { return ds->events[2 + 2 * i]; };
    auto here = [&](int k) { return resident && resident[k]; };   // input already on the device
    std::vector<void*> dptrs(ds->in_stage);
    for (int k = 0; k < p.n_inputs; ++k)
        if (here(k)) dptrs[k] = ptrs[k];
    dptrs.push_back(ds->out_stage);
    int rc = 0;
    auto fail = [&](int code) {
        cudaStreamSynchronize(ds->h2d);
        cudaStreamSynchronize(ds->stream);
        cudaStreamSynchronize(ds->d2h);
        cudaGetLastError();
        return code;
    };

    // inputs every panel reads whole
    for (int k = 0; k < p.n_inputs && !rc; ++k)
        if (p.in_rb[k] == 0 && !here(k))
            rc = copy_async(ds->in_stage[k], ptrs[k], p.in_bytes[k], ds->h2d, "host-to-device copy");
    if (rc) return fail(rc);
    cudaEventRecord(whole, ds->h2d);
    cudaStreamWaitEvent(ds->stream, whole, 0);
    if (ready) cudaStreamWaitEvent(ds->stream, (cudaEvent_t)ready, 0);   // resident inputs filled
    cudaEventRecord(ds->tev[0], ds->stream);
    if ((rc = run_steps(p, ds, ds->device, dptrs.data(), ds->stream, Pass{Pass::Once, 0, 0}))) return fail(rc);
    cudaEventRecord(ds->tev[1], ds->stream);

    for (int i = 0; i < panels; ++i) {
        const int64_t r0 = bounds[i].first, rows = bounds[i].second;
        for (int k = 0; k < p.n_inputs && !rc; ++k) {
            const int64_t b = p.in_rb[k];
            if (b == 0 || here(k)) continue;
            if (p.stream_cols) {
                // columns [r0, r0 + rows) of x (N rows of M elements): one
                // strided copy, the same band in the staged x
                const Step& t = p.steps[0];
                const size_t es = (size_t)t.dst_esize, pitch = (size_t)t.M * es;
                cudaError_t e = cudaMemcpy2DAsync(static_cast<char*>(ds->in_stage[k]) + r0 * es, pitch,
                                                  static_cast<const char*>(ptrs[k]) + r0 * es, pitch, (size_t)rows * es,
                                                  (size_t)t.N, cudaMemcpyDefault, ds->h2d);
                if (e != cudaSuccess) {
                    cudaGetLastError();
                    set_error(7, std::string("host-to-device copy: ") + cudaGetErrorString(e));
                    rc = 7;
                }
                continue;
            }
            rc = copy_async(static_cast<char*>(ds->in_stage[k]) + r0 * b, static_cast<const char*>(ptrs[k]) + r0 * b,
                            rows * b, ds->h2d, "host-to-device copy");
        }
        if (rc) return fail(rc);
        cudaEventRecord(in_done(i), ds->h2d);
        cudaStreamWaitEvent(ds->stream, in_done(i), 0);
        cudaEventRecord(ds->tev[2 + 2 * i], ds->stream);
        if ((rc = run_steps(p, ds, ds->device, dptrs.data(), ds->stream, Pass{Pass::Panel, r0, rows})))
            return fail(rc);
        cudaEventRecord(ds->tev[3 + 2 * i], ds->stream);
        cudaEventRecord(run_done(i), ds->stream);
    }
    for (int i = 0; i < panels; ++i) {
        const int64_t r0 = bounds[i].first, rows = bounds[i].second;
        cudaStreamWaitEvent(ds->d2h, run_done(i), 0);
        if ((rc = copy_async(static_cast<char*>(ptrs[p.n_inputs]) + r0 * p.out_rb,
                             static_cast<char*>(ds->out_stage) + r0 * p.out_rb, rows * p.out_rb, ds->d2h,
                             "device-to-host copy")))
            return fail(rc);
    }
    for (cudaStream_t st : {ds->h2d, ds->stream, ds->d2h})
        if ((rc = sync_stream(st))) return fail(rc);
    p.last_device_ms = timed_ms(ds, (size_t)panels + 1);
    return check_device_error_word(ds->device);
}

}  // namespace

int run_plan_host(Plan& p, void* const* ptrs, int n_ptrs, const unsigned char* resident, void* ready) {
    if (n_ptrs != p.n_inputs + 1) {
        set_error(8, "plan takes " + std::to_string(p.n_inputs + 1) + " pointers, got " + std::to_string(n_ptrs));
        return 8;
    }
    int dev = options().device;
    if (dev < 0) {
        if (cudaGetDevice(&dev) != cudaSuccess) {
            cudaGetLastError();
            set_error(4, "no CUDA device available");
            return 4;
        }
    }
    if (cudaSetDevice(dev) != cudaSuccess) {
        cudaGetLastError();
        set_error(4, "cannot select CUDA device " + std::to_string(dev));
        return 4;
    }
    DeviceState* ds = nullptr;
    if (int rc = ensure_device_state(p, dev, ds)) return rc;
    if (!ds->stream) {
        if (cudaStreamCreateWithFlags(&ds->stream, cudaStreamNonBlocking) != cudaSuccess) {
            cudaGetLastError();
            set_error(6, "cudaStreamCreate failed");
            return 6;
        }
    }
    if (ds->in_stage.size() != (size_t)p.n_inputs) {
        // one device block for the inputs, at the offsets a small call's
        // packed host buffer uses too (one copy moves all of them)
        ds->in_off.assign(p.n_inputs, 0);
        int64_t total = 0;
        for (int k = 0; k < p.n_inputs; ++k) {
            ds->in_off[k] = total;
            total += (p.in_bytes[k] + 255) / 256 * 256;
        }
        if (int rc = alloc(&ds->in_block, total)) return rc;
        ds->in_block_bytes = total;
        ds->in_stage.assign(p.n_inputs, nullptr);
        for (int k = 0; k < p.n_inputs; ++k)
            ds->in_stage[k] = p.in_bytes[k] ? static_cast<char*>(ds->in_block) + ds->in_off[k] : nullptr;
        if (int rc = alloc(&ds->out_stage, p.out_bytes)) return rc;
    }
    if (int rc = ensure_tmps(p, ds)) return rc;
    const int panels = host_panel_count(p);
    if (panels > 1) return run_plan_host_streamed(p, ds, ptrs, panels, resident, ready);
    if (ready) cudaStreamWaitEvent(ds->stream, (cudaEvent_t)ready, 0);   // resident inputs filled
    // Small calls (inputs and output within the pinned buffer, no resident
    // input): every input is copied on the CPU into the pinned buffer at
    // its offset in the device input block, and ONE host-to-device copy
    // moves them all (each copy on the stream costs ~5 us on B200, more
    // than the CPU copy of up to 1 MiB); the output comes back in one copy,
    // through the buffer when the caller's is pageable.  Otherwise operands
    // in pageable memory pass through the pinned buffer one copy each and
    // pinned host or device pointers are copied from directly.
    std::vector<int64_t> stage_off(p.n_inputs + 1, -1);
    bool any_resident = false;
    for (int k = 0; k < p.n_inputs; ++k) any_resident = any_resident || (resident && resident[k]);
    auto pageable = [](const void* q) {
        cudaPointerAttributes a;
        if (cudaPointerGetAttributes(&a, q) != cudaSuccess) { cudaGetLastError(); return false; }
        return a.type == cudaMemoryTypeUnregistered;
    };
    const int64_t out_round = (p.out_bytes + 255) / 256 * 256;
    bool pack_all = !any_resident && ds->in_block_bytes > 0 && ds->in_block_bytes + out_round <= kPackedCallBytes;
    // pinned inputs are packed only while the extra CPU copy is cheap (a
    // few microseconds); pageable ones go through the buffer anyway
    if (pack_all && ds->in_block_bytes > kPackPinnedBytes)
        for (int k = 0; k < p.n_inputs && pack_all; ++k)
            if (p.in_bytes[k] && !pageable(ptrs[k])) pack_all = false;
    {
        int64_t total = 0;
        if (pack_all) {
            // no pointer queries: every input is copied on the CPU, and the
            // output comes back through the buffer too (one small CPU copy)
            for (int k = 0; k < p.n_inputs; ++k) if (p.in_bytes[k]) stage_off[k] = ds->in_off[k];
            total = ds->in_block_bytes;
            if (p.out_bytes) stage_off[p.n_inputs] = total;
            total += out_round;
        } else {
            for (int k = 0; k <= p.n_inputs; ++k) {
                const int64_t b = k < p.n_inputs ? ((resident && resident[k]) ? 0 : p.in_bytes[k]) : p.out_bytes;
                if (b == 0 || !pageable(ptrs[k])) continue;
                stage_off[k] = total;
                total += (b + 255) / 256 * 256;
            }
        }
        bool staged = total > 0 && total <= kPackedCallBytes;
        if (staged && !ds->host_stage) {
            if (cudaHostAlloc(&ds->host_stage, (size_t)kPackedCallBytes, cudaHostAllocDefault) == cudaSuccess) {
                ds->host_stage_bytes = (size_t)kPackedCallBytes;
            } else {
                cudaGetLastError();
                ds->host_stage = nullptr;
                staged = false;   // direct copies instead
            }
        }
        if (!staged) {
            stage_off.assign(p.n_inputs + 1, -1);
            pack_all = false;
        }
    }
    char* const stage = (char*)ds->host_stage;
    auto h2d_failed = [&](cudaError_t e) {
        cudaGetLastError();
        // copies already queued may still read the pinned staging buffer:
        // let them finish before the next call can overwrite it
        cudaStreamSynchronize(ds->stream);
        cudaGetLastError();
        set_error(7, std::string("host-to-device copy: ") + cudaGetErrorString(e));
        return 7;
    };
    // The device error word rides on the same stream into a pinned word --
    // for plans with a tensor-core step, the only kernels whose bounded
    // waits can set it (a word left by an earlier device-resident run is
    // reported by bafe_cuda_synchronize or the next such call).
    const int edev = ds->device;
    bool has_tc = false;
    for (const Step& st : p.steps) has_tc = has_tc || st.kind == StepKind::GemmTc;
    if (has_tc && edev >= 0 && edev < 64 && g_err_word[edev] && !ds->err_host &&
        cudaHostAlloc((void**)&ds->err_host, 4, cudaHostAllocDefault) != cudaSuccess) {
        cudaGetLastError();
        ds->err_host = nullptr;
    }
    const bool err_copy = has_tc && ds->err_host && edev >= 0 && edev < 64 && g_err_word[edev];
    if (int rc = ensure_timing_events(ds, 2)) return rc;
    std::vector<void*> dptrs(ds->in_stage);
    for (int k = 0; k < p.n_inputs; ++k)
        if (resident && resident[k]) dptrs[k] = ptrs[k];
    dptrs.push_back(ds->out_stage);
    const int64_t out_off = stage_off[p.n_inputs];
    // everything after the inputs are in place: the plan, the copy out, the
    // error word (err_async: its copy is queued)
    bool err_async = false;
    bool capturing = false;
    // inside a capture a plain record only marks a dependency; an external
    // record node records the timing event on every replay
    auto record = [&](cudaEvent_t ev) {
        if (capturing) cudaEventRecordWithFlags(ev, ds->stream, cudaEventRecordExternal);
        else cudaEventRecord(ev, ds->stream);
    };
    auto enqueue_rest = [&]() -> int {
        record(ds->tev[0]);
        if (int rc = run_plan_device(p, dptrs.data(), (int)dptrs.size(), ds->stream)) return rc;
        record(ds->tev[1]);
        if (p.out_bytes) {
            void* to = out_off >= 0 ? (void*)(stage + out_off) : ptrs[p.n_inputs];
            cudaError_t e = cudaMemcpyAsync(to, ds->out_stage, (size_t)p.out_bytes, cudaMemcpyDefault, ds->stream);
            if (e != cudaSuccess) {
                cudaGetLastError();
                set_error(7, std::string("device-to-host copy: ") + cudaGetErrorString(e));
                return 7;
            }
        }
        if (err_copy) {
            err_async = cudaMemcpyAsync(ds->err_host, g_err_word[edev], 4, cudaMemcpyDeviceToHost, ds->stream) == cudaSuccess;
            if (!err_async) cudaGetLastError();
        }
        return 0;
    };
    auto enqueue_failed = [&](int rc) {
        // queued copies may still use the pinned buffer: let them finish
        cudaStreamSynchronize(ds->stream);
        cudaGetLastError();
        return rc;
    };
    if (pack_all) {
        for (int k = 0; k < p.n_inputs; ++k)
            if (p.in_bytes[k]) memcpy(stage + stage_off[k], ptrs[k], (size_t)p.in_bytes[k]);
        if (err_copy) *ds->err_host = 0;
        auto enqueue_all = [&]() -> int {
            cudaError_t e = cudaMemcpyAsync(ds->in_block, stage, (size_t)ds->in_block_bytes, cudaMemcpyHostToDevice,
                                            ds->stream);
            if (e != cudaSuccess) {
                cudaGetLastError();
                set_error(7, std::string("host-to-device copy: ") + cudaGetErrorString(e));
                return 7;
            }
            return enqueue_rest();
        };
        // the second packed call of this state captures the sequence as a
        // graph (the first has made every allocation and load); later ones
        // replay it.  A capture that fails leaves the state eager.
        if (!ds->graph_exec && !ds->graph_failed && ds->packed_calls >= 1 && options().host_graphs) {
            const int64_t lc0 = g_launch_count;
            cudaGraph_t graph = nullptr;
            bool ok = cudaStreamBeginCapture(ds->stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
            capturing = ok;
            const int rc = ok ? enqueue_all() : 0;
            capturing = false;
            if (ok) ok = cudaStreamEndCapture(ds->stream, &graph) == cudaSuccess && graph && rc == 0;
            if (ok) ok = cudaGraphInstantiate(&ds->graph_exec, graph, 0) == cudaSuccess;
            if (graph) cudaGraphDestroy(graph);
            ds->graph_kernels = g_launch_count - lc0;
            g_launch_count = lc0;
            if (!ok) {
                cudaGetLastError();
                if (ds->graph_exec) cudaGraphExecDestroy(ds->graph_exec);
                ds->graph_exec = nullptr;
                ds->graph_failed = true;
                clear_error();                           // the call runs eagerly below
            }
        }
        if (ds->graph_exec && options().host_graphs) {
            if (cudaGraphLaunch(ds->graph_exec, ds->stream) != cudaSuccess) {
                cudaGetLastError();
                set_error(7, "cudaGraphLaunch of the host call failed");
                return enqueue_failed(7);
            }
            g_launch_count += ds->graph_kernels;
            err_async = err_copy;
        } else {
            if (int rc = enqueue_all()) return enqueue_failed(rc);
            ++ds->packed_calls;
        }
    } else {
        for (int k = 0; k < p.n_inputs; ++k) {
            if (p.in_bytes[k] == 0 || (resident && resident[k])) continue;
            const void* src = ptrs[k];
            if (stage_off[k] >= 0) {
                memcpy(stage + stage_off[k], ptrs[k], (size_t)p.in_bytes[k]);
                src = stage + stage_off[k];
            }
            cudaError_t e = cudaMemcpyAsync(ds->in_stage[k], src, (size_t)p.in_bytes[k], cudaMemcpyDefault, ds->stream);
            if (e != cudaSuccess) return h2d_failed(e);
        }
        if (err_copy) *ds->err_host = 0;
        if (int rc = enqueue_rest()) return enqueue_failed(rc);
    }
    cudaError_t e = cudaStreamSynchronize(ds->stream);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error(9, std::string("device error: ") + cudaGetErrorString(e));
        return 9;
    }
    if (p.out_bytes && out_off >= 0) memcpy(ptrs[p.n_inputs], stage + out_off, (size_t)p.out_bytes);
    p.last_device_ms = timed_ms(ds, 1);
    if (!has_tc) return 0;
    return err_async ? report_error_word(edev, *ds->err_host) : check_device_error_word(edev);
}

int time_plan_device(Plan& p, void* const* ptrs, int n_ptrs, void* stream_v, int iters, double& ms) {
    ms = -1.0;
    if (iters < 1) iters = 1;
    cudaStream_t st = (cudaStream_t)stream_v;
    if (int rc = run_plan_device(p, ptrs, n_ptrs, st)) return rc;   // untimed: loads, allocates
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (cudaEventCreate(&e0) != cudaSuccess || cudaEventCreate(&e1) != cudaSuccess) {
        cudaGetLastError();
        if (e0) cudaEventDestroy(e0);
        set_error(6, "cudaEventCreate failed");
        return 6;
    }
    int rc = 0;
    cudaEventRecord(e0, st);
    for (int i = 0; i < iters && !rc; ++i) rc = run_plan_device(p, ptrs, n_ptrs, st);
    cudaEventRecord(e1, st);
    cudaError_t e = cudaEventSynchronize(e1);
    float total = 0.0f;
    if (!rc && e != cudaSuccess) {
        cudaGetLastError();
        set_error(9, std::string("device error: ") + cudaGetErrorString(e));
        rc = 9;
    }
    if (!rc && cudaEventElapsedTime(&total, e0, e1) != cudaSuccess) {
        cudaGetLastError();
        set_error(9, "cudaEventElapsedTime failed");
        rc = 9;
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (rc) return rc;
    int dev = 0;
    cudaGetDevice(&dev);
    if ((rc = check_device_error_word(dev))) return rc;
    ms = total / iters;
    return 0;
}

void release_plan_device_state(Plan& p) {
    Driver& d = driver();
    int prev = -1;
    cudaGetDevice(&prev);
    for (DeviceState* s : p.dev) {
        if (!s) continue;
        cudaSetDevice(s->device);
        if (s->stream) cudaStreamSynchronize(s->stream);
        for (void* t : s->tmp) if (t) cudaFree(t);
        if (s->in_block) cudaFree(s->in_block);
        if (s->out_stage) cudaFree(s->out_stage);
        if (s->tc_ws) cudaFree(s->tc_ws);
        if (s->tc_ctr) cudaFree(s->tc_ctr);
        if (s->graph_exec) cudaGraphExecDestroy(s->graph_exec);
        if (s->host_stage) cudaFreeHost(s->host_stage);
        if (s->err_host) cudaFreeHost(s->err_host);
        for (cudaStream_t st : {s->h2d, s->d2h}) if (st) { cudaStreamSynchronize(st); cudaStreamDestroy(st); }
        for (cudaEvent_t ev : s->events) cudaEventDestroy(ev);
        for (cudaEvent_t ev : s->tev) cudaEventDestroy(ev);
        if (s->stream) cudaStreamDestroy(s->stream);
        if (s->module && d.ok) d.moduleUnload(s->module);
        delete s;
    }
    p.dev.clear();
    if (prev >= 0) cudaSetDevice(prev);
    cudaGetLastError();
}

}  // namespace bafe_cuda
