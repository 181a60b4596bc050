// Graph executor: the B200 counterpart of LoadedModel::forward
// (drivers/teeny-cuda/src/model/mod.rs:524-700) for a whole lowered DAG.
//
// The reference walks its DAG per call: it allocates every node's output
// (mem::alloc, :573), launches the node's PTX on the null stream and
// synchronises after each kernel (device/mod.rs:430-485), then frees the
// intermediates.  Here the graph is built once from nodes named after the
// reference's graph ops, shapes are inferred as nodes are added, and
// tb_graph_plan lays every input and intermediate tensor out in one device
// arena by liveness (first fit over [first use, last use] intervals), so a
// run allocates nothing.  A run is the node launches in order on the
// context's stream, with no synchronisation; optionally the launches are
// captured once into a CUDA graph and replayed.  Inputs are written into
// their planned buffers before a run; outputs are read from theirs.
//
// Ops whose graph lowering is a stub or a TODO in the reference
// (kernels/teeny-kernels/src/graph/mod.rs: RmsNorm's RuntimeOp :454,
// RotaryEmbedding :2472, MultiHeadAttention :2477, Gather :2527, ArgMax
// :2250) are node kinds here like the others.
#include <math.h>

#include <algorithm>
#include <vector>

#include "attention.h"
#include "common.cuh"

struct tb_graph {
    struct Tensor {
        int dtype = TB_F32;
        std::vector<int64_t> shape;
        int kind = 2;                  // 0 input, 1 parameter, 2 intermediate
        const void* ext = nullptr;     // parameter: caller's device memory
        size_t bytes = 0, offset = 0;  // planned tensors: offset in the arena
        int first = -1, last = -1;     // node indices of the producer / last consumer
        bool output = false;
        int64_t numel() const {
            int64_t n = 1;
            for (int64_t d : shape) n *= d;
            return n;
        }
    };
    struct Node {
        int op;
        std::vector<int> in;
        int out;
        tb_node_attr attr;
        size_t scratch = 0;   // bytes of per-node scratch (the conv workspace)
    };
    tb_ctx* ctx = nullptr;
    std::vector<Tensor> t;
    std::vector<Node> nodes;
    uint8_t* arena = nullptr;
    size_t arena_bytes = 0, scratch_off = 0;
    bool planned = false;
    int capture = 0;
    cudaStream_t cap_stream = nullptr;
    cudaGraphExec_t exec = nullptr;
};

namespace tb {

static size_t dtype_size(int dt) { return dt == TB_F32 || dt == TB_I32 ? 4 : dt == TB_BF16 ? 2 : 1; }
static size_t align256(size_t b) { return (b + 255) / 256 * 256; }

static const void* cptr(tb_graph* g, int id) {
    const tb_graph::Tensor& x = g->t[id];
    return x.kind == 1 ? x.ext : g->arena + x.offset;
}
static void* mptr(tb_graph* g, int id) { return g->arena + g->t[id].offset; }

// Launches node i (planned graph, arena allocated).
static int run_node(tb_graph* g, int i) {
    tb_ctx* ctx = g->ctx;
    const tb_graph::Node& n = g->nodes[i];
    const tb_node_attr& a = n.attr;
    const tb_graph::Tensor& x = g->t[n.in[0]];
    auto in = [&](int k) -> const void* { return k < (int)n.in.size() && n.in[k] >= 0 ? cptr(g, n.in[k]) : nullptr; };
    const int64_t last = x.shape.back();
    switch (n.op) {
        case TB_G_LINEAR: {
            const int64_t N = g->t[n.in[1]].shape[0];
            const int flags = (in(2) ? TB_EPI_BIAS : 0) | (in(3) ? TB_EPI_RESIDUAL : 0);
            return tb_linear_fwd(ctx, x.dtype, in(0), in(1), (const float*)in(2), in(3), mptr(g, n.out),
                                 x.numel() / last, N, last, flags);
        }
        case TB_G_MATMUL:
            return tb_matmul_fwd(ctx, x.dtype, in(0), in(1), mptr(g, n.out), x.numel() / last,
                                 g->t[n.in[1]].shape[1], last);
        case TB_G_RMSNORM:
            return tb_rmsnorm_fwd(ctx, x.dtype, in(0), in(1), mptr(g, n.out), nullptr, x.numel() / last, last, a.eps);
        case TB_G_LAYERNORM:
            return tb_layernorm_fwd(ctx, x.dtype, in(0), in(1), in(2), mptr(g, n.out), x.numel() / last, last, a.eps);
        case TB_G_ACT: return tb_act_fwd(ctx, a.act, x.dtype, in(0), mptr(g, n.out), x.numel());
        case TB_G_ADD: return tb_add_fwd(ctx, x.dtype, in(0), in(1), mptr(g, n.out), x.numel());
        case TB_G_SWIGLU: return tb_swiglu_fwd(ctx, x.dtype, in(0), in(1), mptr(g, n.out), x.numel());
        case TB_G_ATTENTION: {
            // token-major rows, as the projections write them: q [B, S, Hq * D] and
            // k / v [B, S, Hkv * D], or one fused qkv [B, S, (Hq + 2 Hkv) * D]; the
            // kernels read them (and write O [B, S, Hq * D]) through strides
            const int64_t B = x.shape[0], S = x.shape[1];
            const bool fused = n.in.size() == 1;
            const int64_t D = fused ? last / (a.heads + 2 * a.kv_heads) : last / a.heads;
            const int64_t kv_row = fused ? last : g->t[n.in[1]].shape.back();
            const size_t es = dtype_size(x.dtype);
            AttnTensors at{};
            at.q = in(0);
            at.q_sh = D, at.q_ss = last, at.q_sb = S * last;
            at.k = fused ? (const uint8_t*)in(0) + (size_t)a.heads * D * es : in(1);
            at.v = fused ? (const uint8_t*)in(0) + (size_t)(a.heads + a.kv_heads) * D * es : in(2);
            at.kv_sh = D, at.kv_ss = kv_row, at.kv_sb = S * kv_row;
            at.kv_len_alloc = (int)S;
            at.o = mptr(g, n.out);
            at.o_sh = D, at.o_ss = (int64_t)a.heads * D, at.o_sb = S * a.heads * D;
            at.lse = nullptr;
            if (x.dtype == TB_F32)
                return attn_f32_launch(ctx, at, (int)B, a.heads, a.kv_heads, (int)S, (int)S, (int)D, a.scale, a.causal);
            return attn_tc_launch(ctx, at, (int)B, a.heads, a.kv_heads, (int)S, (int)S, (int)D, a.scale, a.causal);
        }
        case TB_G_ROPE:   // x [T, H, D], positions int32 [T]
            return tb_rope_fwd(ctx, x.dtype, in(0), (const int32_t*)in(1), mptr(g, n.out), x.shape[0],
                               (int)x.shape[1], (int)x.shape[2], a.theta);
        case TB_G_GATHER: {   // table [V, D], ids int32 [...]
            const tb_graph::Tensor& ids = g->t[n.in[1]];
            return tb_embedding_fwd(ctx, x.dtype, in(0), (const int32_t*)in(1), mptr(g, n.out), ids.numel(),
                                    x.shape[1], x.shape[0]);
        }
        case TB_G_ARGMAX:
            return tb_argmax_fwd(ctx, x.dtype, in(0), (int32_t*)mptr(g, n.out), x.numel() / last, last);
        case TB_G_CONV2D: {
            const tb_graph::Tensor& w = g->t[n.in[1]];
            return tb_conv2d_fwd(ctx, x.dtype, in(0), in(1), (const float*)in(2), (const float*)in(3),
                                 (const float*)in(4), mptr(g, n.out), (int)x.shape[0], (int)x.shape[1], (int)w.shape[0],
                                 (int)x.shape[2], (int)x.shape[3], (int)w.shape[2], (int)w.shape[3], a.stride, a.pad,
                                 a.act, g->arena + g->scratch_off, n.scratch);
        }
        case TB_G_BATCHNORM:
            return tb_batchnorm_fwd(ctx, x.dtype, in(0), (const float*)in(1), (const float*)in(2), (const float*)in(3),
                                    (const float*)in(4), mptr(g, n.out), x.shape[0], x.shape[1],
                                    x.numel() / (x.shape[0] * x.shape[1]), a.eps);
        default: return set_error(ctx, TB_ERR_ARG, "graph: node %d has unknown op %d", i, n.op);
    }
}

static int run_nodes(tb_graph* g) {
    for (int i = 0; i < (int)g->nodes.size(); i++) {
        const int rc = run_node(g, i);
        if (rc) return rc;
    }
    return TB_OK;
}

static int add_tensor(tb_graph* g, int dtype, int rank, const int64_t* shape, int kind, const void* ext, int* id) {
    if (!g || !id || rank < 1 || rank > 8 || !shape) return TB_ERR_ARG;
    if (g->planned) return set_error(g->ctx, TB_ERR_ARG, "graph: already planned");
    if (dtype != TB_F32 && dtype != TB_BF16 && dtype != TB_I32)
        return set_error(g->ctx, TB_ERR_UNSUPPORTED, "graph: dtype %d", dtype);
    tb_graph::Tensor t;
    t.dtype = dtype;
    t.shape.assign(shape, shape + rank);
    for (int64_t d : t.shape)
        if (d <= 0) return set_error(g->ctx, TB_ERR_SHAPE, "graph: non-positive dimension");
    t.kind = kind;
    t.ext = ext;
    *id = (int)g->t.size();
    g->t.push_back(t);
    return TB_OK;
}

}  // namespace tb

using namespace tb;

extern "C" {

int tb_graph_create(tb_ctx* ctx, tb_graph** out) {
    if (!ctx || !out) return TB_ERR_ARG;
    tb_graph* g = new tb_graph();
    g->ctx = ctx;
    *out = g;
    return TB_OK;
}

int tb_graph_destroy(tb_graph* g) {
    if (!g) return TB_OK;
    cudaSetDevice(g->ctx->device);
    if (g->exec) cudaGraphExecDestroy(g->exec);
    if (g->cap_stream) cudaStreamDestroy(g->cap_stream);
    if (g->arena) cudaFree(g->arena);
    delete g;
    return TB_OK;
}

int tb_graph_input(tb_graph* g, int dtype, int rank, const int64_t* shape, int* id) {
    return add_tensor(g, dtype, rank, shape, 0, nullptr, id);
}

int tb_graph_param(tb_graph* g, int dtype, int rank, const int64_t* shape, const void* dev_ptr, int* id) {
    if (!dev_ptr) return TB_ERR_ARG;
    return add_tensor(g, dtype, rank, shape, 1, dev_ptr, id);
}

int tb_graph_node(tb_graph* g, int op, const int* inputs, int n_inputs, const tb_node_attr* attr, int* out_id) {
    if (!g || !inputs || n_inputs < 1 || !out_id) return TB_ERR_ARG;
    tb_ctx* ctx = g->ctx;
    if (g->planned) return set_error(ctx, TB_ERR_ARG, "graph: already planned");
    for (int k = 0; k < n_inputs; k++)
        if (inputs[k] >= (int)g->t.size() || (inputs[k] < 0 && k < 2))
            return set_error(ctx, TB_ERR_ARG, "graph: input %d of the node is not a tensor", k);
    tb_node_attr a{};
    if (attr) a = *attr;
    const tb_graph::Tensor& x = g->t[inputs[0]];
    auto T = [&](int k) -> const tb_graph::Tensor& { return g->t[inputs[k]]; };
    std::vector<int64_t> out = x.shape;
    int odt = x.dtype;
    size_t scratch = 0;
    const int64_t last = x.shape.back();
    auto need = [&](bool c, const char* what) {
        if (!c) set_error(ctx, TB_ERR_SHAPE, "graph: %s", what);
        return c;
    };
    switch (op) {
        case TB_G_LINEAR:
            if (!need(n_inputs >= 2 && n_inputs <= 4 && T(1).shape.size() == 2 && T(1).shape[1] == last,
                      "linear: w [N, K] (+ bias [N], residual [.., N])"))
                return TB_ERR_SHAPE;
            out.back() = T(1).shape[0];
            if (n_inputs > 2 && inputs[2] >= 0 && !need(T(2).dtype == TB_F32 && T(2).numel() == out.back(), "linear: f32 bias [N]"))
                return TB_ERR_SHAPE;
            if (n_inputs > 3 && inputs[3] >= 0 &&
                !need(T(3).numel() == x.numel() / last * out.back() && T(3).dtype == x.dtype, "linear: residual [.., N]"))
                return TB_ERR_SHAPE;
            break;
        case TB_G_MATMUL:
            if (!need(n_inputs == 2 && T(1).shape.size() == 2 && T(1).shape[0] == last, "matmul: b [K, N]")) return TB_ERR_SHAPE;
            out.back() = T(1).shape[1];
            break;
        case TB_G_RMSNORM:
            if (!need(n_inputs == 2 && T(1).numel() == last, "rmsnorm: w [N]")) return TB_ERR_SHAPE;
            break;
        case TB_G_LAYERNORM:
            if (!need(n_inputs == 3 && T(1).numel() == last && T(2).numel() == last, "layernorm: w, b [N]")) return TB_ERR_SHAPE;
            break;
        case TB_G_ACT: break;
        case TB_G_ADD:
        case TB_G_SWIGLU:
            if (!need(n_inputs == 2 && T(1).numel() == x.numel(), "elementwise: operand sizes differ")) return TB_ERR_SHAPE;
            break;
        case TB_G_ATTENTION: {
            const bool fused = n_inputs == 1;
            if (!need((n_inputs == 3 || fused) && x.shape.size() == 3 && a.heads > 0 && a.kv_heads > 0 &&
                          a.heads % a.kv_heads == 0,
                      "attention: q, k, v [B, S, heads * D] or one qkv [B, S, (heads + 2 kv_heads) * D]"))
                return TB_ERR_SHAPE;
            const int64_t units = fused ? a.heads + 2 * a.kv_heads : a.heads;
            if (!need(last % units == 0, "attention: row length is not a multiple of the heads")) return TB_ERR_SHAPE;
            const int64_t D = last / units;
            if (!fused && !need(T(1).shape == T(2).shape && T(1).shape.size() == 3 && T(1).shape[0] == x.shape[0] &&
                                    T(1).shape[1] == x.shape[1] && T(1).shape[2] == a.kv_heads * D &&
                                    T(1).dtype == x.dtype && T(2).dtype == x.dtype,
                                "attention: k, v [B, S, kv_heads * D]"))
                return TB_ERR_SHAPE;
            if (!need(x.dtype == TB_F32 ? D <= 128 : (D == 64 || D == 128), "attention: head dim (f32 <= 128, bf16 64 / 128)"))
                return TB_ERR_SHAPE;
            out.back() = a.heads * D;
            if (a.scale == 0.f) a.scale = 1.0f / sqrtf((float)D);
            break;
        }
        case TB_G_ROPE:
            if (!need(n_inputs == 2 && x.shape.size() == 3 && T(1).dtype == TB_I32 && T(1).numel() == x.shape[0],
                      "rope: x [T, H, D], positions int32 [T]"))
                return TB_ERR_SHAPE;
            if (a.theta == 0.f) a.theta = 10000.f;
            break;
        case TB_G_GATHER:
            if (!need(n_inputs == 2 && x.shape.size() == 2 && T(1).dtype == TB_I32, "gather: table [V, D], ids int32"))
                return TB_ERR_SHAPE;
            out = T(1).shape;
            out.push_back(x.shape[1]);
            break;
        case TB_G_ARGMAX:
            out.pop_back();
            if (out.empty()) out.push_back(1);
            odt = TB_I32;
            break;
        case TB_G_CONV2D: {
            if (!need(n_inputs >= 2 && n_inputs <= 5 && x.shape.size() == 4 && T(1).shape.size() == 4 &&
                          T(1).shape[1] == x.shape[1],
                      "conv2d: x [B, C, H, W], w [Co, C, KH, KW] (+ bias, bn scale, bn shift)"))
                return TB_ERR_SHAPE;
            if (a.stride <= 0) a.stride = 1;
            if (a.act == 0 && !attr) a.act = TB_ACT_NONE;
            const int64_t OH = (x.shape[2] + 2 * a.pad - T(1).shape[2]) / a.stride + 1;
            const int64_t OW = (x.shape[3] + 2 * a.pad - T(1).shape[3]) / a.stride + 1;
            if (!need(OH > 0 && OW > 0, "conv2d: output size")) return TB_ERR_SHAPE;
            out = {x.shape[0], T(1).shape[0], OH, OW};
            size_t ws = 0;
            if (tb_conv2d_workspace_size(x.dtype, (int)x.shape[0], (int)x.shape[1], (int)T(1).shape[0], (int)x.shape[2],
                                         (int)x.shape[3], (int)T(1).shape[2], (int)T(1).shape[3], a.stride, a.pad,
                                         &ws) != TB_OK)
                return set_error(ctx, TB_ERR_SHAPE, "graph: conv2d shape");
            scratch = ws;
            break;
        }
        case TB_G_BATCHNORM:
            if (!need(n_inputs == 5 && x.shape.size() >= 2, "batchnorm: x [B, C, ...], gamma, beta, mean, var"))
                return TB_ERR_SHAPE;
            break;
        default: return set_error(ctx, TB_ERR_ARG, "graph: unknown op %d", op);
    }
    int id;
    int rc = add_tensor(g, odt, (int)out.size(), out.data(), 2, nullptr, &id);
    if (rc) return rc;
    tb_graph::Node n;
    n.op = op;
    n.in.assign(inputs, inputs + n_inputs);
    n.out = id;
    n.attr = a;
    n.scratch = scratch;
    g->nodes.push_back(n);
    *out_id = id;
    return TB_OK;
}

int tb_graph_mark_output(tb_graph* g, int id) {
    if (!g || id < 0 || id >= (int)g->t.size()) return TB_ERR_ARG;
    if (g->planned) return set_error(g->ctx, TB_ERR_ARG, "graph: already planned");
    g->t[id].output = true;
    return TB_OK;
}

int tb_graph_plan(tb_graph* g, int capture) {
    if (!g) return TB_ERR_ARG;
    tb_ctx* ctx = g->ctx;
    if (g->planned) return set_error(ctx, TB_ERR_ARG, "graph: already planned");
    const int nn = (int)g->nodes.size();
    // liveness intervals [first, last] in node indices; inputs and outputs
    // (marked, or produced and never consumed) keep their buffers for the whole run
    size_t scratch = 0;
    for (int i = 0; i < nn; i++) {
        const auto& n = g->nodes[i];
        g->t[n.out].first = i;
        g->t[n.out].last = std::max(g->t[n.out].last, i);
        for (int k : n.in)
            if (k >= 0) g->t[k].last = std::max(g->t[k].last, i);
        scratch = std::max(scratch, n.scratch);
    }
    for (auto& t : g->t) {
        if (t.kind == 1) continue;
        t.bytes = align256((size_t)t.numel() * dtype_size(t.dtype));
        const bool consumed = t.kind == 2 ? t.last > t.first : true;
        if (t.kind == 0) t.first = 0;
        if (t.output || !consumed || t.kind == 0) t.last = nn;
    }
    // first fit by decreasing size against the placed tensors whose intervals overlap
    std::vector<int> order;
    for (int i = 0; i < (int)g->t.size(); i++)
        if (g->t[i].kind != 1) order.push_back(i);
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return g->t[a].bytes > g->t[b].bytes; });
    std::vector<int> placed;
    size_t top = 0;
    for (int id : order) {
        tb_graph::Tensor& t = g->t[id];
        std::vector<std::pair<size_t, size_t>> busy;
        for (int p : placed) {
            const tb_graph::Tensor& o = g->t[p];
            if (o.first <= t.last && t.first <= o.last) busy.push_back({o.offset, o.offset + o.bytes});
        }
        std::sort(busy.begin(), busy.end());
        size_t off = 0;
        for (auto& b : busy) {
            if (off + t.bytes <= b.first) break;
            off = std::max(off, b.second);
        }
        t.offset = off;
        top = std::max(top, off + t.bytes);
        placed.push_back(id);
    }
    g->scratch_off = align256(top);
    g->arena_bytes = g->scratch_off + align256(scratch) + 256;
    TB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    if (cudaMalloc(reinterpret_cast<void**>(&g->arena), g->arena_bytes) != cudaSuccess) {
        cudaGetLastError();
        return set_error(ctx, TB_ERR_OOM, "graph: arena of %zu bytes", g->arena_bytes);
    }
    g->capture = capture;
    g->planned = true;
    return TB_OK;
}

int tb_graph_arena_bytes(tb_graph* g, size_t* bytes) {
    if (!g || !bytes || !g->planned) return TB_ERR_ARG;
    *bytes = g->arena_bytes;
    return TB_OK;
}

int tb_graph_tensor_ptr(tb_graph* g, int id, void** ptr) {
    if (!g || !ptr || id < 0 || id >= (int)g->t.size() || !g->planned) return TB_ERR_ARG;
    *ptr = g->t[id].kind == 1 ? const_cast<void*>(g->t[id].ext) : (void*)(g->arena + g->t[id].offset);
    return TB_OK;
}

int tb_graph_write(tb_graph* g, int id, const void* src, size_t bytes) {
    if (!g || !src || id < 0 || id >= (int)g->t.size()) return TB_ERR_ARG;
    tb_ctx* ctx = g->ctx;
    if (!g->planned || g->t[id].kind == 1) return set_error(ctx, TB_ERR_ARG, "graph_write: not a planned tensor");
    const size_t need = (size_t)g->t[id].numel() * dtype_size(g->t[id].dtype);
    TB_REQUIRE(ctx, bytes == need, TB_ERR_SHAPE, "graph_write: %zu bytes for a tensor of %zu", bytes, need);
    TB_CUDA_TRY(ctx, cudaMemcpyAsync(g->arena + g->t[id].offset, src, bytes, cudaMemcpyDefault, ctx->stream));
    return TB_OK;
}

int tb_graph_read(tb_graph* g, int id, void* dst, size_t bytes) {
    if (!g || !dst || id < 0 || id >= (int)g->t.size()) return TB_ERR_ARG;
    tb_ctx* ctx = g->ctx;
    if (!g->planned || g->t[id].kind == 1) return set_error(ctx, TB_ERR_ARG, "graph_read: not a planned tensor");
    const size_t need = (size_t)g->t[id].numel() * dtype_size(g->t[id].dtype);
    TB_REQUIRE(ctx, bytes == need, TB_ERR_SHAPE, "graph_read: %zu bytes for a tensor of %zu", bytes, need);
    TB_CUDA_TRY(ctx, cudaMemcpyAsync(dst, g->arena + g->t[id].offset, bytes, cudaMemcpyDefault, ctx->stream));
    return TB_OK;
}

int tb_graph_run(tb_graph* g) {
    if (!g) return TB_ERR_ARG;
    tb_ctx* ctx = g->ctx;
    if (!g->planned) return set_error(ctx, TB_ERR_ARG, "graph: call tb_graph_plan first");
    if (!g->capture) return run_nodes(g);
    if (!g->exec) {
        // capture the node launches once (ordered after what is already queued)
        TB_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
        if (!g->cap_stream) TB_CUDA_TRY(ctx, cudaStreamCreateWithFlags(&g->cap_stream, cudaStreamNonBlocking));
        cudaStream_t saved = ctx->stream;
        ctx->stream = g->cap_stream;
        cudaGraph_t cg = nullptr;
        cudaError_t e = cudaStreamBeginCapture(g->cap_stream, cudaStreamCaptureModeThreadLocal);
        if (e != cudaSuccess) {
            ctx->stream = saved;
            return set_error(ctx, TB_ERR_CUDA, "graph: begin capture: %s", cudaGetErrorString(e));
        }
        const int rc = run_nodes(g);
        e = cudaStreamEndCapture(g->cap_stream, &cg);
        ctx->stream = saved;
        if (rc) {
            if (cg) cudaGraphDestroy(cg);
            return rc;
        }
        if (e != cudaSuccess) return set_error(ctx, TB_ERR_CUDA, "graph: end capture: %s", cudaGetErrorString(e));
        e = cudaGraphInstantiate(&g->exec, cg, 0);
        cudaGraphDestroy(cg);
        if (e != cudaSuccess) return set_error(ctx, TB_ERR_CUDA, "graph: instantiate: %s", cudaGetErrorString(e));
    }
    TB_CUDA_TRY(ctx, cudaGraphLaunch(g->exec, ctx->stream));
    return TB_OK;
}

}  // extern "C"
