// Stand-in for the Teco-Inference plugin SDK header <plugin/register_op.h>.
//
// The real SDK (TVM + Teco-Inference, libTecoInferPluginUtil.so) is not
// available here, so this header reproduces just the surface the reference's
// plugins are written against (doc/README_PLUGIN.md:52-111 and
// teco/plugin/plugin*/plugin_*.cc):
//   * tvm::AttrsNode / TVM_DECLARE_ATTRS / TVM_ATTR_FIELD / TVM_REGISTER_NODE_TYPE
//     (attribute declarations; values come from OpAttr / ComputeContext);
//   * TECO_INFER::OpAttr::GetAttr<T>(name);
//   * TECO_INFER::ComputeContext with GetInputDataPtr(name or index),
//     GetOutputDataPtr(i), GetAttr(name, value), GetInputShape(name or index, shape)
//     and GetStream();
//   * TECO_INFER::AbstractPluginOp with InferOutputShape and Enqueue;
//   * REGISTER_PLUGIN_OP_IMPL(name, cls) and the PLUGIN_REGISTER_OP(name) spec
//     builder (.Input/.Type/.Desc/.AttrType<>/.Register).
// A plugin written against the real SDK compiles unchanged against this one.
// The library also exports a small C entry (teco_plugin_infer / teco_plugin_enqueue,
// defined in plugin_host.cc) through which tests drive a registered plugin the way
// the engine would.
#ifndef TECOOPS_B200_PLUGIN_STANDIN_REGISTER_OP_H_
#define TECOOPS_B200_PLUGIN_STANDIN_REGISTER_OP_H_

#include <cuda_runtime.h>

#include <cstdint>
#include <functional>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <vector>

// ---- TVM attribute declarations (declarative only in the stand-in) --------------
namespace tvm {
template <typename T>
struct AttrsNode {};
struct AttrFieldStub {
    template <typename V>
    AttrFieldStub &set_default(const V &) { return *this; }
    AttrFieldStub &describe(const char *) { return *this; }
};
}  // namespace tvm
#define TVM_DECLARE_ATTRS(Cls, Name) static constexpr const char *_type_key = Name; \
    template <typename F> void _visit_attrs(F &&)
#define TVM_ATTR_FIELD(f) (void)(f), ::tvm::AttrFieldStub()
#define TVM_REGISTER_NODE_TYPE(Cls) static_assert(sizeof(Cls) > 0, "attrs")

namespace TECO_INFER {

// Attribute values: integer attributes (block sizes, dtypes) and floating ones (eps).
class OpAttr {
 public:
    std::map<std::string, int64_t> ints;
    std::map<std::string, double> floats;
    template <typename T>
    T GetAttr(const std::string &name) const {
        auto f = floats.find(name);
        auto it = ints.find(name);
        if (std::is_floating_point<T>::value && f != floats.end()) return static_cast<T>(f->second);
        if (it != ints.end()) return static_cast<T>(it->second);
        if (f != floats.end()) return static_cast<T>(f->second);
        throw std::runtime_error("plugin attribute missing: " + name);
    }
};

class ComputeContext {
 public:
    std::map<std::string, void *> inputs;
    std::map<std::string, std::vector<int>> shapes;
    std::vector<std::string> input_order;   // inputs by position
    std::vector<void *> outputs;
    OpAttr attr;
    cudaStream_t stream = nullptr;

    void *GetInputDataPtr(const std::string &name) {
        auto it = inputs.find(name);
        return it == inputs.end() ? nullptr : it->second;
    }
    void *GetInputDataPtr(int i) {
        return i >= 0 && i < (int)input_order.size() ? GetInputDataPtr(input_order[i]) : nullptr;
    }
    void GetInputShape(int i, std::vector<int> &shape) {
        if (i >= 0 && i < (int)input_order.size())
            GetInputShape(input_order[i], shape);
        else
            shape.clear();
    }
    void *GetOutputDataPtr(int i) { return i < (int)outputs.size() ? outputs[i] : nullptr; }
    template <typename T>
    void GetAttr(const std::string &name, T &value) { value = attr.GetAttr<T>(name); }
    void GetInputShape(const std::string &name, std::vector<int> &shape) {
        auto it = shapes.find(name);
        shape = it == shapes.end() ? std::vector<int>{} : it->second;
    }
    cudaStream_t GetStream() { return stream; }
};

class AbstractPluginOp {
 public:
    virtual ~AbstractPluginOp() = default;
    virtual void InferOutputShape(const std::vector<std::vector<int>> &total_input_shape,
                                  int n_input, std::vector<std::vector<int>> &total_output_shape,
                                  int n_output, const OpAttr &attr) = 0;
    virtual void Enqueue(std::shared_ptr<ComputeContext> &ctx) = 0;
};

struct PluginSpec {
    std::string name;
    std::vector<std::string> inputs;
};

// registries (one instance per process, inline so every translation unit shares it)
inline std::map<std::string, std::function<std::unique_ptr<AbstractPluginOp>()>> &
plugin_impls() {
    static std::map<std::string, std::function<std::unique_ptr<AbstractPluginOp>()>> m;
    return m;
}
inline std::map<std::string, PluginSpec> &plugin_specs() {
    static std::map<std::string, PluginSpec> m;
    return m;
}

class PluginSpecBuilder {
 public:
    explicit PluginSpecBuilder(const char *name) { spec_.name = name; }
    PluginSpecBuilder &Input(const char *n) {
        spec_.inputs.push_back(n);
        return *this;
    }
    PluginSpecBuilder &Type(const char *) { return *this; }
    PluginSpecBuilder &Desc(const char *) { return *this; }
    template <typename A>
    PluginSpecBuilder &AttrType() { return *this; }
    int Register() {
        plugin_specs()[spec_.name] = spec_;
        return 0;
    }

 private:
    PluginSpec spec_;
};

}  // namespace TECO_INFER

#define TECO_PLUGIN_CAT2(a, b) a##b
#define TECO_PLUGIN_CAT(a, b) TECO_PLUGIN_CAT2(a, b)
#define REGISTER_PLUGIN_OP_IMPL(name, Cls)                                              \
    static const int TECO_PLUGIN_CAT(_teco_plugin_impl_, name) = [] {                  \
        ::TECO_INFER::plugin_impls()[#name] = [] {                                      \
            return std::unique_ptr<::TECO_INFER::AbstractPluginOp>(new Cls());          \
        };                                                                              \
        return 0;                                                                       \
    }();
#define PLUGIN_REGISTER_OP(name) \
    static const int TECO_PLUGIN_CAT(_teco_plugin_spec_, __LINE__) = ::TECO_INFER::PluginSpecBuilder(name)

#endif  // TECOOPS_B200_PLUGIN_STANDIN_REGISTER_OP_H_
