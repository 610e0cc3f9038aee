// api.cpp -- the extern "C" surface of libbafe_cuda.so (include/bafe_cuda.h):
// plan cache keyed by graph hash, host-function trampolines, stats, options.
#include "internal.h"

#include <cuda_runtime.h>

#include <array>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>

#define BAFE_API extern "C" __attribute__((visibility("default")))

namespace bafe_cuda {

Options& options() {
    static Options o;
    static bool init = false;
    if (!init) {
        init = true;
        if (const char* p = getenv("BAFE_GEMM_PRECISION")) o.gemm_precision = p;
        if (const char* d = getenv("BAFE_DEVICE")) o.device = atoi(d);
        if (const char* t = getenv("BAFE_TC_PAIR")) o.tc_pair = atoi(t) != 0;
        if (const char* h = getenv("BAFE_HOST_PANELS")) o.host_panels = strcmp(h, "auto") == 0 ? -1 : atoi(h);
        if (const char* c = getenv("BAFE_TC_CONVERT")) o.tc_convert = strcmp(c, "auto") == 0 ? -1 : (atoi(c) != 0);
        if (const char* f = getenv("BAFE_KSLICE_FREE_SMS")) o.kslice_free_sms = atoi(f) > 0 ? atoi(f) : 0;
        if (const char* hg = getenv("BAFE_HOST_GRAPHS")) o.host_graphs = atoi(hg) != 0;
    }
    return o;
}

namespace {

std::recursive_mutex g_mu;
std::vector<Plan*> g_plans;                 // plan id -> plan (nullptr once dropped)
std::map<std::string, int> g_by_key;        // plan key -> plan id
bafe_jit_stats g_stats = {0, 0, 0, 0};

// ------------------------------------------------------- trampolines --
// The legacy kernel ABI has no context argument (jit.h:26-35): the caller
// gets a bare function pointer and calls f(in_0, ..., in_{n-1}, out).  Each
// live plan is therefore bound to one of kSlots distinct functions; the
// function reads the first n+1 pointer arguments (n = the plan's input
// count, at most kMaxArgs-1) and runs the plan on them.  Plans with more
// inputs are bound to the same slot in a second bank of functions that take
// kMaxArgsWide pointers, so that a function never reads many more argument
// slots than its caller passes.
constexpr int kSlots = 256;          // the reference caches 256 kernels (jit.c:164)
constexpr int kMaxArgs = 17;         // 16 inputs + out
constexpr int kMaxArgsWide = 65;     // 64 inputs + out
int g_slot_plan[kSlots];
bool g_slots_init = false;

int run_slot(int slot, void** a);

template <int S>
void trampoline(void* p0, void* p1, void* p2, void* p3, void* p4, void* p5, void* p6, void* p7, void* p8,
                void* p9, void* p10, void* p11, void* p12, void* p13, void* p14, void* p15, void* p16) {
    void* a[kMaxArgs] = {p0, p1, p2, p3, p4, p5, p6, p7, p8, p9, p10, p11, p12, p13, p14, p15, p16};
    run_slot(S, a);
}
typedef void (*TrampolineFn)(void*, void*, void*, void*, void*, void*, void*, void*, void*, void*, void*, void*,
                             void*, void*, void*, void*, void*);

template <size_t... I>
constexpr std::array<TrampolineFn, sizeof...(I)> make_trampolines(std::index_sequence<I...>) {
    return {{&trampoline<(int)I>...}};
}
const std::array<TrampolineFn, kSlots> kTrampolines = make_trampolines(std::make_index_sequence<kSlots>{});

template <size_t>
using ArgPtr = void*;
template <int S, class Seq>
struct WideTrampoline;
template <int S, size_t... I>
struct WideTrampoline<S, std::index_sequence<I...>> {
    static void fn(ArgPtr<I>... p) {
        void* a[sizeof...(I)] = {p...};
        run_slot(S, a);
    }
};
template <int S>
using WideOf = WideTrampoline<S, std::make_index_sequence<kMaxArgsWide>>;
typedef decltype(&WideOf<0>::fn) WideFn;
template <size_t... I>
constexpr std::array<WideFn, sizeof...(I)> make_wide_trampolines(std::index_sequence<I...>) {
    return {{&WideOf<(int)I>::fn...}};
}
const std::array<WideFn, kSlots> kWideTrampolines = make_wide_trampolines(std::make_index_sequence<kSlots>{});

// The function handed out for a slot: the narrow bank up to 16 inputs.
bafe_kernel_fn slot_function(int slot, int n_inputs) {
    return n_inputs <= kMaxArgs - 1 ? reinterpret_cast<bafe_kernel_fn>(kTrampolines[slot])
                                    : reinterpret_cast<bafe_kernel_fn>(kWideTrampolines[slot]);
}
// Slot of a handed-out function, either bank; -1 if it is none of them.
int slot_of_function(bafe_kernel_fn fn) {
    for (int i = 0; i < kSlots; ++i)
        if (reinterpret_cast<bafe_kernel_fn>(kTrampolines[i]) == fn ||
            reinterpret_cast<bafe_kernel_fn>(kWideTrampolines[i]) == fn)
            return i;
    return -1;
}

void init_slots() {
    if (g_slots_init) return;
    for (int i = 0; i < kSlots; ++i) g_slot_plan[i] = -1;
    g_slots_init = true;
}

int slot_of_plan(int plan_id) {
    for (int i = 0; i < kSlots; ++i)
        if (g_slot_plan[i] == plan_id) return i;
    return -1;
}

int run_slot(int slot, void** a) {
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    int pid = g_slot_plan[slot];
    if (pid < 0 || pid >= (int)g_plans.size() || !g_plans[pid]) {
        set_error(10, "stale kernel function: its plan was dropped by bafe_cuda_jit_clear or invalidate");
        return 10;
    }
    Plan& p = *g_plans[pid];
    return run_plan_host(p, a, p.n_inputs + 1);
}

void drop_all_plans() {
    for (Plan* p : g_plans) {
        if (!p) continue;
        release_plan_device_state(*p);
        delete p;
    }
    g_plans.clear();
    g_by_key.clear();
    init_slots();
    for (int i = 0; i < kSlots; ++i) g_slot_plan[i] = -1;
}

Plan* plan_ptr(int id) {
    if (id < 0 || id >= (int)g_plans.size()) return nullptr;
    return g_plans[id];
}

void write_err(char* buf, size_t n, const std::string& msg) {
    if (buf && n > 0) snprintf(buf, n, "%s", msg.c_str());
}

}  // namespace

std::recursive_mutex& api_mutex() { return g_mu; }
Plan* find_plan(int id) { return plan_ptr(id); }
int plan_id_of(bafe_kernel_fn fn) {
    if (!fn) return -1;
    init_slots();
    const int slot = slot_of_function(fn);
    return slot < 0 ? -1 : g_slot_plan[slot];
}
void drop_memory_cache() { drop_all_plans(); }

}  // namespace bafe_cuda

using namespace bafe_cuda;

BAFE_API int bafe_cuda_version(void) { return 1000; }

BAFE_API int bafe_cuda_jit_hash_graph(const bafe_graph* g, char* out, size_t out_size) {
    return hash_graph(g, out, out_size);
}

BAFE_API bafe_kernel_fn bafe_cuda_jit_get_or_compile(const bafe_graph* g, char* err_buf, size_t err_buf_size) {
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    init_slots();
    if (err_buf && err_buf_size) err_buf[0] = '\0';
    char hash[65];
    if (hash_graph(g, hash, sizeof(hash)) < 0) {
        write_err(err_buf, err_buf_size, "hash failed");
        return nullptr;
    }
    const Options& opt = options();
    std::string key = std::string(hash) + "|prec=" + opt.gemm_precision + (opt.tc_pair ? "|pair" : "|single") +
                      "|conv=" + std::to_string(opt.tc_convert);
    auto it = g_by_key.find(key);
    if (it != g_by_key.end() && plan_ptr(it->second)) {
        int slot = slot_of_plan(it->second);
        if (slot >= 0) {
            g_stats.hits++;
            return slot_function(slot, plan_ptr(it->second)->n_inputs);
        }
    }
    g_stats.misses++;
    Graph G;
    std::string err;
    if (parse_graph(g, G, err) != 0) {
        write_err(err_buf, err_buf_size, err);
        set_error(2, err);
        g_stats.compile_failures++;
        return nullptr;
    }
    if ((int)G.inputs.size() > kMaxArgsWide - 1) {
        err = "graph has more than 64 inputs (the kernel function takes at most 65 pointers)";
        write_err(err_buf, err_buf_size, err);
        set_error(2, err);
        g_stats.compile_failures++;
        return nullptr;
    }
    Plan* p = new Plan();
    p->graph_hash = hash;
    p->key = key;
    if (lower_graph(G, opt, *p, err) != 0) {
        write_err(err_buf, err_buf_size, err);
        set_error(2, err);
        g_stats.compile_failures++;
        delete p;
        return nullptr;
    }
    bool from_cache = false;
    if (compile_cubin(p->source, p->source_hash, p->cubin, from_cache, err) != 0) {
        write_err(err_buf, err_buf_size, err);
        set_error(3, err);
        g_stats.compile_failures++;
        delete p;
        return nullptr;
    }
    if (from_cache) g_stats.hits++;   // on-disk hit, counted like jit.c:241
    else g_stats.compiles++;
    int slot = slot_of_plan(-1);
    if (slot < 0) {
        // The reference stops caching after 256 kernels (jit.c:320); a
        // context-free function needs a slot, so evict the oldest plan.
        int victim = -1;
        for (int i = 0; i < (int)g_plans.size(); ++i)
            if (g_plans[i] && slot_of_plan(i) >= 0) { victim = i; break; }
        if (victim >= 0) {
            slot = slot_of_plan(victim);
            g_by_key.erase(g_plans[victim]->key);
            release_plan_device_state(*g_plans[victim]);
            delete g_plans[victim];
            g_plans[victim] = nullptr;
            g_slot_plan[slot] = -1;
        }
    }
    if (slot < 0) {
        write_err(err_buf, err_buf_size, "no free kernel slot");
        delete p;
        return nullptr;
    }
    p->id = (int)g_plans.size();
    g_plans.push_back(p);
    g_by_key[key] = p->id;
    g_slot_plan[slot] = p->id;
    return slot_function(slot, p->n_inputs);
}

BAFE_API void bafe_cuda_jit_set_cache_dir(const char* dir) {
    if (!dir) return;
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    set_cache_dir(dir);
}

BAFE_API const char* bafe_cuda_jit_cache_dir(void) {
    static std::string s;
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    s = cache_dir();
    return s.c_str();
}

BAFE_API bafe_jit_stats bafe_cuda_jit_get_stats(void) { return g_stats; }

BAFE_API void bafe_cuda_jit_clear(void) {
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    drop_all_plans();
    g_stats = {0, 0, 0, 0};
}

BAFE_API void bafe_cuda_jit_invalidate_memory_cache(void) {
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    drop_all_plans();
}

BAFE_API int bafe_cuda_plan_of(bafe_kernel_fn fn) {
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    init_slots();
    const int slot = slot_of_function(fn);
    return slot < 0 ? -1 : g_slot_plan[slot];
}

BAFE_API int bafe_cuda_plan_num_inputs(int plan) {
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    Plan* p = plan_ptr(plan);
    return p ? p->n_inputs : -1;
}

BAFE_API int bafe_cuda_plan_describe(int plan, char* buf, size_t buf_size) {
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    Plan* p = plan_ptr(plan);
    std::string s = p ? p->describe : std::string();
    if (buf && buf_size) snprintf(buf, buf_size, "%s", s.c_str());
    return (int)s.size();
}

BAFE_API int64_t bafe_cuda_plan_output_bytes(int plan) {
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    Plan* p = plan_ptr(plan);
    return p ? p->out_bytes : -1;
}

BAFE_API int64_t bafe_cuda_plan_input_bytes(int plan, int i) {
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    Plan* p = plan_ptr(plan);
    if (!p || i < 0 || i >= p->n_inputs) return -1;
    return p->in_bytes[i];
}

BAFE_API int bafe_cuda_plan_row_split(int plan, int64_t* rows, int64_t* in_row_bytes, int n_inputs,
                                      int64_t* out_row_bytes) {
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    Plan* p = plan_ptr(plan);
    if (!p) return -1;
    if (rows) *rows = p->stream_ok ? p->stream_rows : 0;
    if (out_row_bytes) *out_row_bytes = p->stream_ok ? p->out_rb : 0;
    for (int k = 0; in_row_bytes && k < n_inputs && k < p->n_inputs; ++k)
        in_row_bytes[k] = p->stream_ok ? p->in_rb[k] : 0;
    return p->stream_ok ? 1 : 0;
}

BAFE_API int bafe_cuda_run_device(int plan, void* const* ptrs, int n_ptrs, void* stream) {
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    Plan* p = plan_ptr(plan);
    if (!p) { set_error(10, "unknown plan " + std::to_string(plan)); return 10; }
    return run_plan_device(*p, ptrs, n_ptrs, stream);
}

BAFE_API int bafe_cuda_plan_num_steps(int plan) {
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    Plan* p = plan_ptr(plan);
    if (!p) { set_error(10, "unknown plan " + std::to_string(plan)); return -1; }
    return (int)p->steps.size();
}

BAFE_API int bafe_cuda_run_device_timed(int plan, void* const* ptrs, int n_ptrs, void* stream, void* const* step_events,
                                        int n_events) {
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    Plan* p = plan_ptr(plan);
    if (!p) { set_error(10, "unknown plan " + std::to_string(plan)); return 10; }
    return run_plan_device_timed(*p, ptrs, n_ptrs, stream, step_events, n_events);
}

BAFE_API int bafe_cuda_plan_k_slice_align(int plan) {
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    Plan* p = plan_ptr(plan);
    if (!p) { set_error(10, "unknown plan " + std::to_string(plan)); return -1; }
    return plan_k_slice_align(*p);
}

BAFE_API int bafe_cuda_run_device_ksliced(int plan, void* const* ptrs, int n_ptrs, void* stream, int n_slices,
                                          const int64_t* k_bounds, void* const* ready) {
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    Plan* p = plan_ptr(plan);
    if (!p) { set_error(10, "unknown plan " + std::to_string(plan)); return 10; }
    return run_plan_device_ksliced(*p, ptrs, n_ptrs, stream, n_slices, k_bounds, ready);
}

BAFE_API int bafe_cuda_run_host(int plan, void* const* ptrs, int n_ptrs) {
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    Plan* p = plan_ptr(plan);
    if (!p) { set_error(10, "unknown plan " + std::to_string(plan)); return 10; }
    return run_plan_host(*p, ptrs, n_ptrs);
}

BAFE_API int bafe_cuda_run_host_resident(int plan, void* const* ptrs, int n_ptrs, const unsigned char* resident,
                                         void* ready) {
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    Plan* p = plan_ptr(plan);
    if (!p) { set_error(10, "unknown plan " + std::to_string(plan)); return 10; }
    return run_plan_host(*p, ptrs, n_ptrs, resident, ready);
}

BAFE_API int bafe_cuda_last_error(char* buf, size_t buf_size) {
    std::string msg;
    int code = get_error(msg);
    if (buf && buf_size) snprintf(buf, buf_size, "%s", msg.c_str());
    return code;
}

BAFE_API void bafe_cuda_clear_error(void) { clear_error(); }

BAFE_API int bafe_cuda_set_option(const char* key, const char* value) {
    if (!key || !value) return -1;
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    Options& o = options();
    std::string k = key, v = value;
    if (k == "gemm_precision") {
        if (v != "auto" && v != "3xtf32" && v != "tf32" && v != "exact") return -1;
        o.gemm_precision = v;
        return 0;
    }
    if (k == "tc_pair") {
        if (v != "0" && v != "1") return -1;
        o.tc_pair = v == "1";
        return 0;
    }
    if (k == "tc_convert") {
        if (v != "auto" && v != "0" && v != "1") return -1;
        o.tc_convert = v == "auto" ? -1 : (v == "1");
        return 0;
    }
    if (k == "host_graphs") {
        if (v != "0" && v != "1") return -1;
        o.host_graphs = v == "1";
        return 0;
    }
    if (k == "kslice_free_sms") {
        char* end = nullptr;
        long n = strtol(value, &end, 10);
        if (!end || *end || n < 0 || n > 1024) return -1;
        o.kslice_free_sms = (int)n;
        return 0;
    }
    if (k == "host_panels") {
        if (v == "auto") { o.host_panels = -1; return 0; }
        char* end = nullptr;
        long n = strtol(value, &end, 10);
        if (!end || *end || n < 0 || n > 4096) return -1;
        o.host_panels = (int)n;
        return 0;
    }
    if (k == "device") {
        char* end = nullptr;
        long d = strtol(value, &end, 10);
        if (!end || *end || d < -1) return -1;
        o.device = (int)d;
        return 0;
    }
    return -1;
}

BAFE_API int bafe_cuda_get_option(const char* key, char* buf, size_t buf_size) {
    if (!key) return -1;
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    Options& o = options();
    std::string k = key, v;
    if (k == "gemm_precision") v = o.gemm_precision;
    else if (k == "device") v = std::to_string(o.device);
    else if (k == "tc_pair") v = o.tc_pair ? "1" : "0";
    else if (k == "tc_convert") v = o.tc_convert < 0 ? "auto" : (o.tc_convert ? "1" : "0");
    else if (k == "host_panels") v = o.host_panels < 0 ? "auto" : std::to_string(o.host_panels);
    else if (k == "kslice_free_sms") v = std::to_string(o.kslice_free_sms);
    else if (k == "host_graphs") v = o.host_graphs ? "1" : "0";
    else return -1;
    if (buf && buf_size) snprintf(buf, buf_size, "%s", v.c_str());
    return 0;
}

BAFE_API int64_t bafe_cuda_launch_count(void) { return g_launch_count; }

BAFE_API int64_t bafe_cuda_abi_size(int which) {
    switch (which) {
        case 0: return (int64_t)sizeof(bafe_graph);
        case 1: return (int64_t)sizeof(bafe_node);
        case 2: return (int64_t)sizeof(bafe_op_attrs);
        case 3: return (int64_t)sizeof(bafe_shape);
    }
    return -1;
}

BAFE_API int bafe_cuda_synchronize(void) {
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    return synchronize_current_device();
}
