// ref_harness.cu -- C-ABI shim around the reference CUDA filter.
//
// TEST INFRASTRUCTURE ONLY.  It is compiled, together with the unmodified
// reference source permutohedral.cu, into oracle/_ref/libplattice_ref.so by
// oracle/Makefile, and is loaded only by the tests, the golden-vector script
// and the reference arm of the benchmark.
//
// The reference's own host layer (permuto.cpp:51-69) allocates its workspace
// internally and throws it away, so the lattice it builds cannot be inspected.
// This shim calls the same entry points (permutohedral.cu:685 permuto_filter,
// permutohedral.cu:717 permuto_filter_grad) with caller-owned workspace
// buffers, sized exactly as permuto.cpp:51-69 sizes them, so that the caller
// can read the hash table keys and the per-slot (index, weight) matrix after
// the call.  Every call synchronises and reports the CUDA status, which the
// reference never checks.
#include <cuda_runtime.h>
#include <cstddef>

void permuto_filter(float* weight_out, float* out, const float* values, const float* features,
                    void* matrix_storage, float* h_values_dev, float* blur_values_dev,
                    int* h_entries_dev, signed short* h_keys_dev, int* blur_neighbors_dev,
                    int pd, int vd, int w, int h);
void permuto_filter_grad(float* out, const float* grad_values, const float* weight_in,
                         const float* features, void* matrix_storage, float* h_values_dev,
                         float* blur_values_dev, int* h_entries_dev, signed short* h_keys_dev,
                         int* blur_neighbors_dev, int pd, int vd, int w, int h);

extern "C" {

// Workspace sizes in bytes for n = h*w pixels, as permuto.cpp:51-69.
// sizes[0] matrix, [1] values, [2] blur_values, [3] entries, [4] keys, [5] blur_neighbors
void ref_workspace_sizes(long long n, int pd, int vd, long long* sizes) {
    const long long cap = n * (pd + 1);
    sizes[0] = cap * 8;
    sizes[1] = cap * (vd + 1) * 4;
    sizes[2] = cap * (vd + 1) * 4;
    sizes[3] = cap * 2 * 4;
    sizes[4] = cap * pd * 2;
    sizes[5] = cap * (pd + 1) * 2 * 4;
}

static int ref_status() {
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaGetLastError();
    return (int)e;
}

int ref_forward(float* weight_out, float* out, const float* values, const float* features,
                void* matrix, float* vals, float* blur_vals, int* entries, short* keys,
                int* nbrs, int pd, int vd, int w, int h, int sync) {
    permuto_filter(weight_out, out, values, features, matrix, vals, blur_vals, entries,
                   (signed short*)keys, nbrs, pd, vd, w, h);
    return sync ? ref_status() : (int)cudaGetLastError();
}

int ref_backward(float* grad_out, const float* grad, const float* weight_in, const float* features,
                 void* matrix, float* vals, float* blur_vals, int* entries, short* keys,
                 int* nbrs, int pd, int vd, int w, int h, int sync) {
    permuto_filter_grad(grad_out, grad, weight_in, features, matrix, vals, blur_vals, entries,
                        (signed short*)keys, nbrs, pd, vd, w, h);
    return sync ? ref_status() : (int)cudaGetLastError();
}

}  // extern "C"
