// C entry points of the stand-in plugin host: what the Teco-Inference engine does
// with a registered AbstractPluginOp (shape inference, then Enqueue on its stream),
// exposed so that tests can drive the plugins without the engine.
#include <plugin/register_op.h>

#include <cstring>
#include <exception>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

namespace {
std::string g_last_error;

// attribute values arrive as doubles: integral ones are stored as both kinds
TECO_INFER::OpAttr make_attr(int n_attr, const char *const *names, const double *vals) {
    TECO_INFER::OpAttr a;
    for (int i = 0; i < n_attr; ++i) {
        a.floats[names[i]] = vals[i];
        if (vals[i] == (double)(long long)vals[i]) a.ints[names[i]] = (long long)vals[i];
    }
    return a;
}

std::vector<std::vector<int>> make_shapes(int n, const int *ranks, const int *dims_flat) {
    std::vector<std::vector<int>> s(n);
    int off = 0;
    for (int i = 0; i < n; ++i) {
        s[i].assign(dims_flat + off, dims_flat + off + ranks[i]);
        off += ranks[i];
    }
    return s;
}
}  // namespace

extern "C" {

const char *teco_plugin_last_error() { return g_last_error.c_str(); }

// Registered plugin ops with their declared inputs, "op:in1,in2;op2:..." (returns length).
int teco_plugin_list(char *buf, int cap) {
    std::string s;
    for (auto &kv : TECO_INFER::plugin_specs()) {
        if (!s.empty()) s += ";";
        s += kv.first + ":";
        for (size_t i = 0; i < kv.second.inputs.size(); ++i)
            s += (i ? "," : "") + kv.second.inputs[i];
    }
    if (buf && cap > 0) {
        std::strncpy(buf, s.c_str(), cap - 1);
        buf[cap - 1] = 0;
    }
    return (int)s.size();
}

// InferOutputShape of n_out outputs: returns 0 and fills out_ranks[o] and
// out_dims[8 * o + d] (<= 8 dims each).
int teco_plugin_infer(const char *op, int n_in, const int *ranks, const int *dims_flat,
                      int n_attr, const char *const *attr_names, const double *attr_vals,
                      int n_out, int *out_ranks, int *out_dims) {
    auto it = TECO_INFER::plugin_impls().find(op);
    if (it == TECO_INFER::plugin_impls().end()) return -1;
    try {
        auto impl = it->second();
        std::vector<std::vector<int>> outs(n_out);
        impl->InferOutputShape(make_shapes(n_in, ranks, dims_flat), n_in, outs, n_out,
                               make_attr(n_attr, attr_names, attr_vals));
        for (int o = 0; o < n_out; ++o) {
            out_ranks[o] = (int)outs[o].size();
            for (int i = 0; i < out_ranks[o] && i < 8; ++i) out_dims[8 * o + i] = outs[o][i];
        }
        return 0;
    } catch (const std::exception &e) {
        g_last_error = e.what();
        return -2;
    }
}

namespace {

// Enqueue of `impl` with named inputs on `stream` (a cudaStream_t).
int enqueue_impl(TECO_INFER::AbstractPluginOp &impl, int n_in, const char *const *in_names,
                 void *const *in_ptrs, const int *ranks, const int *dims_flat, int n_out,
                 void *const *out_ptrs, int n_attr, const char *const *attr_names,
                 const double *attr_vals, void *stream) {
    try {
        auto ctx = std::make_shared<TECO_INFER::ComputeContext>();
        auto shapes = make_shapes(n_in, ranks, dims_flat);
        for (int i = 0; i < n_in; ++i) {
            ctx->inputs[in_names[i]] = in_ptrs[i];
            ctx->shapes[in_names[i]] = shapes[i];
            ctx->input_order.push_back(in_names[i]);
        }
        ctx->outputs.assign(out_ptrs, out_ptrs + n_out);
        ctx->attr = make_attr(n_attr, attr_names, attr_vals);
        ctx->stream = static_cast<cudaStream_t>(stream);
        impl.Enqueue(ctx);
        return 0;
    } catch (const std::exception &e) {
        g_last_error = e.what();
        return -2;
    }
}

// op instances that live across Enqueue calls, as an engine keeps one per graph node
std::mutex g_instances_mutex;
std::map<int, std::unique_ptr<TECO_INFER::AbstractPluginOp>> g_instances;
int g_next_instance = 1;

}  // namespace

// One-shot Enqueue: a fresh instance of `op` for this call only (destroyed after it).
int teco_plugin_enqueue(const char *op, int n_in, const char *const *in_names,
                        void *const *in_ptrs, const int *ranks, const int *dims_flat, int n_out,
                        void *const *out_ptrs, int n_attr, const char *const *attr_names,
                        const double *attr_vals, void *stream) {
    auto it = TECO_INFER::plugin_impls().find(op);
    if (it == TECO_INFER::plugin_impls().end()) return -1;
    auto impl = it->second();
    return enqueue_impl(*impl, n_in, in_names, in_ptrs, ranks, dims_flat, n_out, out_ptrs,
                        n_attr, attr_names, attr_vals, stream);
}

// A persistent instance of `op`: returns its id (> 0), or -1 for an unknown op.
int teco_plugin_create(const char *op) {
    auto it = TECO_INFER::plugin_impls().find(op);
    if (it == TECO_INFER::plugin_impls().end()) return -1;
    std::lock_guard<std::mutex> lock(g_instances_mutex);
    const int id = g_next_instance++;
    g_instances[id] = it->second();
    return id;
}

// Enqueue on a persistent instance (the call returns as soon as the work is enqueued).
int teco_plugin_enqueue_instance(int id, int n_in, const char *const *in_names,
                                 void *const *in_ptrs, const int *ranks, const int *dims_flat,
                                 int n_out, void *const *out_ptrs, int n_attr,
                                 const char *const *attr_names, const double *attr_vals,
                                 void *stream) {
    TECO_INFER::AbstractPluginOp *impl = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_instances_mutex);
        auto it = g_instances.find(id);
        if (it == g_instances.end()) return -1;
        impl = it->second.get();
    }
    return enqueue_impl(*impl, n_in, in_names, in_ptrs, ranks, dims_flat, n_out, out_ptrs,
                        n_attr, attr_names, attr_vals, stream);
}

int teco_plugin_destroy(int id) {
    std::lock_guard<std::mutex> lock(g_instances_mutex);
    return g_instances.erase(id) == 1 ? 0 : -1;
}

}  // extern "C"
