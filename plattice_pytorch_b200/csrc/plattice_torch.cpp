// plattice_torch.cpp -- PermutoLatticeFunction (the reference's autograd
// Function, plattice.py:7-19) as a C++ autograd Function, built as the torch
// extension module plattice_pytorch_b200._plattice_torch.
//
// It does what the Python Function does -- the input checks and messages of
// permuto.cpp:33-40,72-85,113-132, the forward through plattice_forward, the
// lattice kept on the autograd context for the backward, the backward
// through plattice_backward on the caller's current stream, no gradient for
// the features -- without the Python interpreter between the autograd engine
// and the library: about 35 us less host time per forward + backward, which
// is most of what a small image costs.
//
// The library's entry points come from the already-loaded
// libplattice_b200.so (set_entry_points, called with their addresses by the
// Python package), so that the process has one copy of the library and of its
// call graphs and status ring.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <array>
#include <map>
#include <mutex>
#include <string>

namespace {

typedef int (*ForwardFn)(float*, float*, const float*, const float*, void*, size_t, void*, size_t, int, int, int,
                         int, void*);
typedef int (*BackwardFn)(float*, const float*, const float*, const float*, void*, size_t, int, void*, size_t, int,
                          int, int, int, void*);
typedef int (*SizesFn)(int, int, int, int, size_t*, size_t*);
typedef int (*ReuseFn)(int, int, int, int, int, size_t*);
typedef const char* (*StringFn)(int);
typedef const char* (*DetailFn)(void);

struct Entry {
    ForwardFn forward = nullptr;
    BackwardFn backward = nullptr;
    SizesFn sizes = nullptr;
    ReuseFn reuse = nullptr;
    StringFn error_string = nullptr;
    DetailFn detail = nullptr;
} g_fn;

void set_entry_points(int64_t fwd, int64_t bwd, int64_t sizes, int64_t reuse, int64_t err, int64_t detail) {
    g_fn.forward = reinterpret_cast<ForwardFn>(fwd);
    g_fn.backward = reinterpret_cast<BackwardFn>(bwd);
    g_fn.sizes = reinterpret_cast<SizesFn>(sizes);
    g_fn.reuse = reinterpret_cast<ReuseFn>(reuse);
    g_fn.error_string = reinterpret_cast<StringFn>(err);
    g_fn.detail = reinterpret_cast<DetailFn>(detail);
}

std::string failure(const char* call, int rc, int h, int w, int pd, int vd) {
    return std::string(call) + " failed: " + g_fn.error_string(rc) + " (status " + std::to_string(rc) + "); h=" +
           std::to_string(h) + " w=" + std::to_string(w) + " pd=" + std::to_string(pd) + " vd=" +
           std::to_string(vd) + "; " + g_fn.detail();
}

struct Sizes {
    size_t lattice, scratch, reuse;
};

// workspace sizes per shape (the library's sizing, cached)
Sizes sizes_of(int h, int w, int pd, int vd) {
    static std::mutex mu;
    static std::map<std::array<int, 4>, Sizes> cache;
    const std::array<int, 4> key{h, w, pd, vd};
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    Sizes s{0, 0, 0};
    int rc = g_fn.sizes(h, w, pd, vd, &s.lattice, &s.scratch);
    TORCH_CHECK(rc == 0, failure("plattice_workspace_sizes", rc, h, w, pd, vd));
    rc = g_fn.reuse(1, h, w, pd, vd, &s.reuse);
    TORCH_CHECK(rc == 0, failure("plattice_reuse_scratch_size", rc, h, w, pd, vd));
    cache.emplace(key, s);
    return s;
}

// CHECK_CUDA / CHECK_CONTIGUOUS of permuto.cpp:33-35
void check_input(const at::Tensor& t, const char* name) {
    TORCH_CHECK(t.is_cuda(), name, " must be CUDA");
    TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

// permuto.cpp:37-40
void check_dims(int64_t pd, int64_t vd) {
    TORCH_CHECK(1 <= pd && pd <= 16, "feature dimension pd must be in [1, 16]");
    TORCH_CHECK(1 <= vd && vd <= 8, "value dimension vd must be in [1, 8]");
}

using torch::autograd::AutogradContext;
using torch::autograd::variable_list;

struct PermutoLatticeFn : public torch::autograd::Function<PermutoLatticeFn> {
    // keep: the lattice stays on the context for the backward; otherwise
    // nothing is kept and the backward rebuilds it, as the reference does
    static at::Tensor forward(AutogradContext* ctx, const at::Tensor& features, const at::Tensor& values,
                              bool keep) {
        TORCH_CHECK(g_fn.forward, "the plattice library's entry points are not set");
        check_input(features, "features");
        check_input(values, "values");
        TORCH_CHECK(features.dim() == 3, "features must be [H, W, pd]");
        TORCH_CHECK(values.dim() == 3, "values must be [H, W, vd]");
        TORCH_CHECK(features.scalar_type() == at::kFloat, "features must be float32");
        TORCH_CHECK(values.scalar_type() == at::kFloat, "values must be float32");
        TORCH_CHECK(features.size(0) == values.size(0) && features.size(1) == values.size(1),
                    "features and values must have matching H, W");
        check_dims(features.size(2), values.size(2));
        TORCH_CHECK(values.device() == features.device(), "features and values must be on the same device");
        const int h = (int)features.size(0), w = (int)features.size(1);
        const int pd = (int)features.size(2), vd = (int)values.size(2);
        const c10::cuda::CUDAGuard guard(features.device());
        const auto opts = features.options();
        at::Tensor out = at::empty({h, w, vd}, opts);
        at::Tensor weight = at::empty({h, w, 1}, opts);
        const Sizes s = sizes_of(h, w, pd, vd);
        at::Tensor lattice = at::empty({(int64_t)s.lattice}, opts.dtype(at::kByte));
        {
            at::Tensor scratch = at::empty({(int64_t)s.scratch}, opts.dtype(at::kByte));
            const int rc = g_fn.forward(weight.data_ptr<float>(), out.data_ptr<float>(), values.data_ptr<float>(),
                                        features.data_ptr<float>(), lattice.data_ptr(), s.lattice,
                                        scratch.data_ptr(), s.scratch, pd, vd, w, h,
                                        at::cuda::getCurrentCUDAStream(features.device().index()).stream());
            TORCH_CHECK(rc == 0, failure("plattice_forward", rc, h, w, pd, vd));
        }
        ctx->save_for_backward({weight, features});
        ctx->saved_data["keep"] = keep;
        if (keep) ctx->saved_data["lattice"] = lattice;
        ctx->saved_data["used"] = false;
        return out;
    }

    // value gradient on the kept lattice (the reference rebuilds it,
    // permutohedral.cu:615-635, as this does when the forward kept nothing);
    // no gradient for the features (plattice.py:19)
    static variable_list backward(AutogradContext* ctx, variable_list grads) {
        const auto saved = ctx->get_saved_variables();
        const at::Tensor& weight = saved[0];
        const at::Tensor& features = saved[1];
        const at::Tensor grad = grads[0].contiguous();
        check_input(grad, "grad_values");
        TORCH_CHECK(grad.dim() == 3, "grad_values must be [H, W, vd]");
        TORCH_CHECK(grad.scalar_type() == at::kFloat, "grad_values must be float32");
        TORCH_CHECK(features.size(0) == grad.size(0) && features.size(1) == grad.size(1),
                    "features and grad_values must have matching H, W");
        check_dims(features.size(2), grad.size(2));
        TORCH_CHECK(grad.device() == features.device(),
                    "features, grad_values and weight_saved must be on the same device");
        const int h = (int)features.size(0), w = (int)features.size(1);
        const int pd = (int)features.size(2), vd = (int)grad.size(2);
        const c10::cuda::CUDAGuard guard(features.device());
        const auto opts = features.options();
        const bool keep = ctx->saved_data["keep"].toBool();
        const bool used = ctx->saved_data["used"].toBool();
        const Sizes s = sizes_of(h, w, pd, vd);
        // kept: the lattice and the reuse scratch (state 1, or 2 after an
        // earlier backward); else a lattice built here (state 0), full scratch
        at::Tensor lattice =
            keep ? ctx->saved_data["lattice"].toTensor() : at::empty({(int64_t)s.lattice}, opts.dtype(at::kByte));
        const int state = keep ? (used ? 2 : 1) : 0;
        const size_t sbytes = keep ? s.reuse : s.scratch;
        at::Tensor grad_values = at::empty({h, w, vd}, opts);
        {
            at::Tensor scratch = at::empty({(int64_t)sbytes}, opts.dtype(at::kByte));
            const int rc = g_fn.backward(grad_values.data_ptr<float>(), grad.data_ptr<float>(),
                                         weight.data_ptr<float>(), features.data_ptr<float>(), lattice.data_ptr(),
                                         (size_t)lattice.numel(), state, scratch.data_ptr(), sbytes, pd, vd, w, h,
                                         at::cuda::getCurrentCUDAStream(features.device().index()).stream());
            // a failed call may have stopped part way: a later backward on
            // this graph rebuilds the lattice instead of reusing it
            if (rc != 0) ctx->saved_data["keep"] = false;
            TORCH_CHECK(rc == 0, failure("plattice_backward", rc, h, w, pd, vd));
        }
        ctx->saved_data["used"] = true;
        return {at::Tensor(), grad_values, at::Tensor()};
    }
};

at::Tensor permuto_lattice(const at::Tensor& features, const at::Tensor& values, bool keep) {
    return PermutoLatticeFn::apply(features, values, keep);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.doc() = "PermutoLatticeFunction as a C++ autograd Function over libplattice_b200.so";
    m.def("set_entry_points", &set_entry_points,
          "addresses of plattice_forward, plattice_backward, plattice_workspace_sizes, "
          "plattice_reuse_scratch_size, plattice_error_string, plattice_last_error_detail");
    m.def("permuto_lattice", &permuto_lattice,
          "forward of PermutoLatticeFunction (out); backward by autograd, on the kept lattice (keep) or on one "
          "rebuilt there",
          py::arg("features"), py::arg("values"), py::arg("keep") = true, py::call_guard<py::gil_scoped_release>());
}
