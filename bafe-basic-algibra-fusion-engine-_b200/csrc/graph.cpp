// graph.cpp -- validation and typing of BAFE's graph struct, graph hash,
// SHA-256.
#include "internal.h"

#include <cstring>
#include <cstdio>

namespace bafe_cuda {

// ------------------------------------------------------------- SHA-256 --
// FIPS 180-4 SHA-256 (a published standard; the round constants are the
// standard's).  Used for the graph hash (the reference keys its cache with
// SHA-256 too, jit.c:131-154) and for the cubin cache key.

namespace {
struct Sha256 {
    uint32_t h[8];
    uint64_t bits = 0;
    uint8_t block[64];
    size_t fill = 0;

    static uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

    Sha256() {
        static const uint32_t iv[8] = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                                       0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};
        memcpy(h, iv, sizeof(h));
    }
    void compress(const uint8_t* p) {
        static const uint32_t K[64] = {
            0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u, 0xab1c5ed5u,
            0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u,
            0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,
            0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u,
            0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u,
            0xa2bfe8a1u, 0xa81a664bu, 0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,
            0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
            0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u};
        uint32_t w[64];
        for (int t = 0; t < 16; ++t)
            w[t] = (uint32_t)p[4 * t] << 24 | (uint32_t)p[4 * t + 1] << 16 |
                   (uint32_t)p[4 * t + 2] << 8 | (uint32_t)p[4 * t + 3];
        for (int t = 16; t < 64; ++t) {
            uint32_t s0 = rotr(w[t - 15], 7) ^ rotr(w[t - 15], 18) ^ (w[t - 15] >> 3);
            uint32_t s1 = rotr(w[t - 2], 17) ^ rotr(w[t - 2], 19) ^ (w[t - 2] >> 10);
            w[t] = w[t - 16] + s0 + w[t - 7] + s1;
        }
        uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
        for (int t = 0; t < 64; ++t) {
            uint32_t t1 = hh + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + K[t] + w[t];
            uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
            hh = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
        }
        h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
    }
    void update(const void* data, size_t len) {
        const uint8_t* p = static_cast<const uint8_t*>(data);
        bits += (uint64_t)len * 8;
        while (len) {
            size_t take = 64 - fill;
            if (take > len) take = len;
            memcpy(block + fill, p, take);
            fill += take; p += take; len -= take;
            if (fill == 64) { compress(block); fill = 0; }
        }
    }
    std::string hex() {
        uint64_t total = bits;
        uint8_t pad = 0x80;
        update(&pad, 1);
        uint8_t zero = 0;
        while (fill != 56) update(&zero, 1);
        uint8_t len[8];
        for (int i = 0; i < 8; ++i) len[i] = (uint8_t)(total >> (56 - 8 * i));
        update(len, 8);
        static const char* digits = "0123456789abcdef";
        std::string s(64, '0');
        for (int i = 0; i < 8; ++i)
            for (int b = 0; b < 4; ++b) {
                uint8_t byte = (uint8_t)(h[i] >> (24 - 8 * b));
                s[8 * i + 2 * b] = digits[byte >> 4];
                s[8 * i + 2 * b + 1] = digits[byte & 15];
            }
        return s;
    }
};
}  // namespace

std::string sha256_hex(const void* data, size_t len) {
    Sha256 s;
    s.update(data, len);
    return s.hex();
}

// Graph hash: the byte stream the reference hashes (jit.c:131-154), field by
// field, raw struct bytes included, so that identical graphs get identical
// keys under both backends.
int hash_graph(const bafe_graph* g, char* out, size_t out_size) {
    if (!g || !out || out_size < 65) return -1;
    Sha256 s;
    s.update(&g->n_inputs, sizeof(g->n_inputs));
    s.update(&g->n_outputs, sizeof(g->n_outputs));
    s.update(&g->n_nodes, sizeof(g->n_nodes));
    const int nn = g->n_nodes < 0 ? 0 : (g->n_nodes > BAFE_MAX_NODES ? BAFE_MAX_NODES : g->n_nodes);
    for (int i = 0; i < nn; ++i) {
        const bafe_node* n = &g->nodes[i];
        const char* op = n->op_name ? n->op_name : "";
        s.update(op, strlen(op) + 1);
        s.update(&n->attrs, sizeof(n->attrs));
        s.update(&n->n_children, sizeof(n->n_children));
        int nc = n->n_children < 0 ? 0 : (n->n_children > BAFE_MAX_CHILDREN ? BAFE_MAX_CHILDREN : n->n_children);
        s.update(n->children, sizeof(bafe_node_id) * (size_t)nc);
        s.update(&n->shape, sizeof(n->shape));
        s.update(&n->dtype, sizeof(n->dtype));
        s.update(&n->layout, sizeof(n->layout));
        if (n->is_input) {
            size_t len = strnlen(n->input_name, BAFE_MAX_ATTR_LEN);
            s.update(n->input_name, len);
            uint8_t z = 0;
            s.update(&z, 1);
        }
        if (n->is_constant) s.update(&n->const_value, sizeof(n->const_value));
    }
    std::string h = s.hex();
    memcpy(out, h.c_str(), 65);
    return 0;
}

// --------------------------------------------------------------- dtypes --

int dtype_size(int dtype) {
    switch (dtype) {
        case BAFE_DTYPE_F32: return 4;
        case BAFE_DTYPE_F64: return 8;
        case BAFE_DTYPE_I32: return 4;
        case BAFE_DTYPE_I64: return 8;
        case BAFE_DTYPE_F16: return 2;
        case BAFE_DTYPE_BF16: return 2;
    }
    return 0;
}

int compute_dtype(int dtype) {
    return (dtype == BAFE_DTYPE_F16 || dtype == BAFE_DTYPE_BF16) ? BAFE_DTYPE_F32 : dtype;
}

const char* dtype_ctype(int dtype) {
    switch (dtype) {
        case BAFE_DTYPE_F32: return "float";
        case BAFE_DTYPE_F64: return "double";
        case BAFE_DTYPE_I32: return "i32";
        case BAFE_DTYPE_I64: return "i64";
        case BAFE_DTYPE_F16: return "u16";
        case BAFE_DTYPE_BF16: return "u16";
    }
    return "void";
}

std::string Shape::str() const {
    std::string s = "(";
    for (int i = 0; i < rank; ++i) {
        if (i) s += ",";
        s += std::to_string((long long)d[i]);
    }
    if (rank == 1) s += ",";
    return s + ")";
}

// ---------------------------------------------------------------- parse --

static Op op_from_name(const char* s) {
    struct { const char* n; Op op; } table[] = {
        {"input", Op::Input}, {"constant", Op::Constant}, {"matmul", Op::MatMul},
        {"add", Op::Add}, {"sub", Op::Sub}, {"mul", Op::Mul}, {"bias_add", Op::BiasAdd},
        {"relu", Op::Relu}, {"neg", Op::Neg}, {"sigmoid", Op::Sigmoid}, {"tanh", Op::Tanh},
        {"transpose", Op::Transpose}, {"reduce_sum", Op::ReduceSum},
        {"reduce_max", Op::ReduceMax}, {"reshape", Op::Reshape},
        {"broadcast_to", Op::BroadcastTo}, {"layout_transform", Op::LayoutTransform},
        {"fused_matmul_relu", Op::FusedMatmulRelu}, {"fused_matmul_bias", Op::FusedMatmulBias},
        {"fused_matmul_bias_relu", Op::FusedMatmulBiasRelu},
        {"fused_bias_relu", Op::FusedBiasRelu},
    };
    for (auto& e : table)
        if (strcmp(e.n, s) == 0) return e.op;
    return Op::Unknown;   // e.g. "scale": the emitter zero-fills (codegen.c:529-533)
}

int parse_graph(const bafe_graph* g, Graph& out, std::string& err) {
    if (!g) { err = "null graph"; return 1; }
    if (g->n_nodes <= 0 || g->n_nodes > BAFE_MAX_NODES) { err = "graph has no nodes"; return 1; }
    if (g->n_outputs <= 0) { err = "graph has no outputs"; return 1; }
    if (g->n_inputs < 0 || g->n_inputs > BAFE_MAX_NODES) { err = "bad input count"; return 1; }
    out.nodes.assign(g->n_nodes, Node());
    for (int i = 0; i < g->n_nodes; ++i) {
        const bafe_node& s = g->nodes[i];
        Node& n = out.nodes[i];
        n.id = i;
        if (!s.op_name) { err = "node " + std::to_string(i) + " has no op name"; return 1; }
        n.opname = s.op_name;
        n.op = s.is_input ? Op::Input : (s.is_constant ? Op::Constant : op_from_name(s.op_name));
        if (s.n_children < 0 || s.n_children > BAFE_MAX_CHILDREN) {
            err = "node " + std::to_string(i) + " has a bad child count"; return 1;
        }
        for (int c = 0; c < s.n_children; ++c) {
            int ch = s.children[c];
            if (ch < 0 || ch >= g->n_nodes || ch == i) {
                err = "node " + std::to_string(i) + " has an out-of-range child"; return 1;
            }
            n.ch.push_back(ch);
        }
        if (s.shape.rank < 0 || s.shape.rank > BAFE_MAX_RANK) {
            err = "node " + std::to_string(i) + " has a bad rank"; return 1;
        }
        n.shape.rank = s.shape.rank;
        for (int d = 0; d < s.shape.rank; ++d) {
            if (s.shape.dims[d] < 0) { err = "node " + std::to_string(i) + " has a negative dim"; return 1; }
            n.shape.d[d] = s.shape.dims[d];
        }
        if (dtype_size((int)s.dtype) == 0) { err = "node " + std::to_string(i) + " has an unknown dtype"; return 1; }
        n.dtype = (int)s.dtype;
        n.layout = (int)s.layout;
        n.name.assign(s.input_name, strnlen(s.input_name, BAFE_MAX_ATTR_LEN));
        for (int k = 0; k < s.attrs.n_perm && k < BAFE_MAX_ATTR_LEN; ++k) n.perm.push_back(s.attrs.perm[k]);
        for (int k = 0; k < s.attrs.n_axes && k < BAFE_MAX_ATTR_LEN; ++k) n.axes.push_back(s.attrs.axes[k]);
        for (int k = 0; k < s.attrs.n_shape && k < BAFE_MAX_ATTR_LEN; ++k) n.tshape.push_back(s.attrs.shape[k]);
        n.keepdims = s.attrs.keepdims;
    }
    out.inputs.clear();
    for (int k = 0; k < g->n_inputs; ++k) {
        int id = g->inputs[k];
        if (id < 0 || id >= g->n_nodes || !g->nodes[id].is_input) {
            err = "graph input " + std::to_string(k) + " is not an input node"; return 1;
        }
        out.nodes[id].input_index = k;
        out.inputs.push_back(id);
    }
    out.root = g->outputs[0];
    if (out.root < 0 || out.root >= g->n_nodes) { err = "output node out of range"; return 1; }
    // The DAG must be acyclic: every child id checked above; detect cycles.
    std::vector<int> state(out.nodes.size(), 0);
    std::vector<std::pair<int, size_t>> st;
    st.push_back({out.root, 0});
    while (!st.empty()) {
        auto& top = st.back();
        int id = top.first;
        if (top.second == 0) {
            if (state[id] == 2) { st.pop_back(); continue; }
            state[id] = 1;
        }
        if (top.second < out.nodes[id].ch.size()) {
            int c = out.nodes[id].ch[top.second++];
            if (state[c] == 1) { err = "graph has a cycle"; return 1; }
            if (state[c] == 0) st.push_back({c, 0});
        } else {
            state[id] = 2;
            st.pop_back();
        }
    }
    return 0;
}

}  // namespace bafe_cuda
