// memcpy_interpose.cpp -- opt-in interposer of cudaMemcpyAsync
// (libsecure_infer_interpose.so), the CUDA form of the reference's
// interposed vendor copy (aclrtMemcpyAsync, secure_infer.cpp:7729-7855).
//
// LD_PRELOADed with SECURE_INFER_INTERPOSE=1, it makes an unmodified caller
// that moves KV blocks with plain cudaMemcpyAsync (vLLM's swap_blocks, a
// torch copy_) take the authenticated path for copies that touch a registered
// host range:
//   host -> device from a registered range  -> secure_infer_h2d_submit
//   device -> host into a registered range  -> secure_infer_d2h_submit
// Everything else -- and every copy when SECURE_INFER_INTERPOSE is not 1 --
// goes to the next cudaMemcpyAsync in the lookup order (the CUDA runtime the
// caller links dynamically).  libsecure_infer.so links its own runtime
// statically, so the library's internal copies never come back here.
//
// As with the reference's hook, H2D copies inside a
// secure_infer_h2d_layer_group_begin/end bracket are batched per layer and
// authenticated by secure_infer_recovery_wait_layer_authentication; D2H copies
// are verified and decrypted by host workers and joined by secure_infer_d2h_wait
// (or the D2H batch bracket).  A registered copy that the library refuses (no
// session, bad arguments) fails with cudaErrorInvalidValue rather than falling
// back to a plain copy.  Only the two explicit directions are interposed;
// cudaMemcpyDefault and the per-thread-stream variants pass through.
#include <cuda_runtime_api.h>
#include <dlfcn.h>

#include <cstdlib>
#include <cstring>

extern "C" int secure_infer_h2d_submit(void* dst, size_t dst_capacity, const void* src, size_t count, void* stream);
extern "C" int secure_infer_d2h_submit(void* dst_host, const void* src_device, size_t count, void* stream);
extern "C" int secure_infer_is_registered_host_range(const void* ptr, size_t bytes);

namespace {

using MemcpyAsyncFn = cudaError_t (*)(void*, const void*, size_t, cudaMemcpyKind, cudaStream_t);

MemcpyAsyncFn next_memcpy_async()
{
    static MemcpyAsyncFn fn = reinterpret_cast<MemcpyAsyncFn>(dlsym(RTLD_NEXT, "cudaMemcpyAsync"));
    return fn;
}

bool interposing()
{
    static const bool on = [] {
        const char* v = std::getenv("SECURE_INFER_INTERPOSE");
        return v != nullptr && std::strcmp(v, "1") == 0;
    }();
    return on;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) cudaError_t cudaMemcpyAsync(void* dst, const void* src, size_t count,
                                                                             cudaMemcpyKind kind, cudaStream_t stream)
{
    if (interposing() && count != 0 && dst != nullptr && src != nullptr) {
        if (kind == cudaMemcpyHostToDevice && secure_infer_is_registered_host_range(src, count) == 1)
            return secure_infer_h2d_submit(dst, count, src, count, stream) == 0 ? cudaSuccess : cudaErrorInvalidValue;
        if (kind == cudaMemcpyDeviceToHost && secure_infer_is_registered_host_range(dst, count) == 1)
            return secure_infer_d2h_submit(dst, src, count, stream) == 0 ? cudaSuccess : cudaErrorInvalidValue;
    }
    const MemcpyAsyncFn next = next_memcpy_async();
    return next != nullptr ? next(dst, src, count, kind, stream) : cudaErrorInitializationError;
}
