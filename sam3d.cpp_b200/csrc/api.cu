// Context management and status reporting for the s3dsp C ABI.
#include <mutex>

#include "s3dsp_internal.h"

using namespace s3dsp;

namespace s3dsp {
namespace {
std::mutex g_pool_mu;
cudaMemPool_t g_pools[64] = {};
}  // namespace

cudaError_t lib_pool(int device, cudaMemPool_t* out) {
    if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_pool_mu);
    if (!g_pools[device]) {
        cudaMemPoolProps props = {};
        props.allocType = cudaMemAllocationTypePinned;
        props.handleTypes = cudaMemHandleTypeNone;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = device;
        cudaMemPool_t pool;
        cudaError_t e = cudaMemPoolCreate(&pool, &props);
        if (e != cudaSuccess) return e;
        uint64_t keep = ~0ull;
        e = cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
        // no reuse of a block freed on another stream whose free has not run
        // yet: the pool would make this stream wait for that one, and contexts
        // on separate streams would serialise on each other's scratch
        int no_deps = 0;
        if (e == cudaSuccess)
            e = cudaMemPoolSetAttribute(pool, cudaMemPoolReuseAllowInternalDependencies, &no_deps);
        if (e != cudaSuccess) {
            cudaMemPoolDestroy(pool);
            return e;
        }
        g_pools[device] = pool;
    }
    *out = g_pools[device];
    return cudaSuccess;
}
}  // namespace s3dsp

extern "C" S3DSP_API uint32_t s3dsp_abi_version(void) { return 1u; }

extern "C" S3DSP_API s3d_status s3dsp_context_create(int32_t device, void* stream, uint32_t flags,
                                                     s3dsp_context** out, char* error,
                                                     uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!out) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "out is NULL");
    *out = nullptr;
    int count = 0;
    S3DSP_CUDA(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
    if (device < 0 || device >= count)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "device %d out of range [0,%d)",
                    device, count);
    S3DSP_CUDA(cudaSetDevice(device), "cudaSetDevice");
    cudaDeviceProp prop;
    S3DSP_CUDA(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
    if (prop.major != 10)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT,
                    "device %d is sm_%d%d; this library is built for sm_100a only", device,
                    prop.major, prop.minor);
    auto* ctx = new (std::nothrow) s3dsp_context();
    if (!ctx) return fail(error, error_capacity, S3D_OUT_OF_MEMORY, "context allocation");
    ctx->device = device;
    ctx->flags = flags;
    ctx->sm_count = prop.multiProcessorCount;
    ctx->sm_device = prop.multiProcessorCount;
    if (!(flags & S3DSP_CONTEXT_OWN_STREAM)) {
        ctx->stream = (cudaStream_t)stream;  // NULL = the legacy default stream
    } else {
        cudaError_t e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
        if (e != cudaSuccess) {
            delete ctx;
            return cuda_fail(error, error_capacity, e, "cudaStreamCreate");
        }
        ctx->owns_stream = true;
    }
    // the library's private pool (the host's default pool keeps its policy)
    cudaMemPool_t pool;
    cudaError_t e = lib_pool(device, &pool);
    if (e != cudaSuccess) {
        s3dsp_context_free(ctx);
        return cuda_fail(error, error_capacity, e, "library memory pool");
    }
    e = cudaMalloc(&ctx->d_status, 4 * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMemsetAsync(ctx->d_status, 0, 4 * sizeof(uint32_t), ctx->stream);
    if (e != cudaSuccess) {
        s3dsp_context_free(ctx);
        return cuda_fail(error, error_capacity, e, "status buffer");
    }
    if (flags & S3DSP_CONTEXT_COPY_STREAMS) {
        // two more non-blocking streams and the slot events; the slots' device
        // buffers are allocated by the first call that uses each slot
        ctx->pipe = new (std::nothrow) s3dsp_host_pipe();
        if (!ctx->pipe) {
            s3dsp_context_free(ctx);
            return fail(error, error_capacity, S3D_OUT_OF_MEMORY, "context allocation");
        }
        s3dsp_host_pipe* p = ctx->pipe;
        e = cudaStreamCreateWithFlags(&p->copy_in, cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&p->copy_out, cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->order, cudaEventDisableTiming);
        for (auto& s : p->slots) {
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s.in_done, cudaEventDisableTiming);
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s.comp_done, cudaEventDisableTiming);
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s.out_done, cudaEventDisableTiming);
        }
        if (e != cudaSuccess) {
            s3dsp_context_free(ctx);
            return cuda_fail(error, error_capacity, e, "copy streams");
        }
    }
    *out = ctx;
    return S3D_OK;
}

extern "C" S3DSP_API void s3dsp_context_free(s3dsp_context* ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    if (s3dsp_host_pipe* p = ctx->pipe) {
        if (p->copy_in) cudaStreamSynchronize(p->copy_in);
        if (p->copy_out) cudaStreamSynchronize(p->copy_out);
        for (auto& s : p->slots) {
            // pool memory: freed (and synchronised) on the copy-in stream, which allocated it
            if (s.d_coords) cudaFreeAsync(s.d_coords, p->copy_in);
            if (s.d_x) cudaFreeAsync(s.d_x, p->copy_in);
            if (s.d_out) cudaFreeAsync(s.d_out, p->copy_in);
            if (s.in_done) cudaEventDestroy(s.in_done);
            if (s.comp_done) cudaEventDestroy(s.comp_done);
            if (s.out_done) cudaEventDestroy(s.out_done);
        }
        if (p->copy_in) {
            cudaStreamSynchronize(p->copy_in);
            cudaStreamDestroy(p->copy_in);
        }
        if (p->copy_out) cudaStreamDestroy(p->copy_out);
        if (p->order) cudaEventDestroy(p->order);
        delete p;
    }
    if (ctx->d_status) cudaFree(ctx->d_status);
    if (ctx->owns_stream && ctx->stream) cudaStreamDestroy(ctx->stream);
    delete ctx;
}

namespace s3dsp {
cudaError_t pipe_join(s3dsp_context* ctx) {
    s3dsp_host_pipe* p = ctx->pipe;
    if (!p) return cudaSuccess;
    // one event, recorded and waited on in turn: a wait uses the record made before it
    cudaError_t e = cudaEventRecord(p->order, p->copy_in);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(ctx->stream, p->order, 0);
    if (e == cudaSuccess) e = cudaEventRecord(p->order, p->copy_out);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(ctx->stream, p->order, 0);
    return e;
}
}  // namespace s3dsp

extern "C" S3DSP_API s3d_status s3dsp_context_fork(s3dsp_context* ctx, char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "ctx is NULL");
    s3dsp_host_pipe* p = ctx->pipe;
    if (!p) return S3D_OK;
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    S3DSP_CUDA(cudaEventRecord(p->order, ctx->stream), "cudaEventRecord");
    S3DSP_CUDA(cudaStreamWaitEvent(p->copy_in, p->order, 0), "cudaStreamWaitEvent");
    S3DSP_CUDA(cudaStreamWaitEvent(p->copy_out, p->order, 0), "cudaStreamWaitEvent");
    return S3D_OK;
}

extern "C" S3DSP_API s3d_status s3dsp_context_join(s3dsp_context* ctx, char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "ctx is NULL");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    S3DSP_CUDA(pipe_join(ctx), "join copy streams");
    return S3D_OK;
}

extern "C" S3DSP_API void* s3dsp_context_stream(const s3dsp_context* ctx) {
    return ctx ? (void*)ctx->stream : nullptr;
}

extern "C" S3DSP_API s3d_status s3dsp_context_set_sm_limit(s3dsp_context* ctx, int32_t sms, char* error,
                                                          uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "ctx is NULL");
    if (sms < 0) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "negative SM limit %d", sms);
    ctx->sm_count = (sms == 0 || sms > ctx->sm_device) ? ctx->sm_device : sms;
    return S3D_OK;
}

namespace s3dsp {
s3d_status check_status(s3dsp_context* ctx, char* error, uint64_t error_capacity) {
    uint32_t st[4] = {0, 0, 0, 0};
    S3DSP_CUDA(cudaMemcpyAsync(st, ctx->d_status, sizeof(st), cudaMemcpyDeviceToHost, ctx->stream),
               "status readback");
    S3DSP_CUDA(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    if (st[0] == 0) return S3D_OK;
    S3DSP_CUDA(cudaMemsetAsync(ctx->d_status, 0, sizeof(st), ctx->stream), "status reset");
    if (st[0] & kErrCoordRange)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT,
                    "coordinate outside the supported domain (0 <= batch < 32768, "
                    "-32768 <= x,y,z < 32768)");
    if (st[0] & kErrDuplicate)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT,
                    "duplicate coordinate (%u rows repeat an earlier row)", st[1]);
    if (st[0] & kErrHashFull)
        return fail(error, error_capacity, S3D_INTERNAL_ERROR, "coordinate hash probe bound exceeded");
    if (st[0] & kErrRowRange)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT,
                    "a row index passed in (upsample / composition rows) is outside its input table");
    if (st[0] & kErrPipelineTimeout)
        return fail(error, error_capacity, S3D_INTERNAL_ERROR,
                    "a device pipeline wait timed out (kernel aborted)");
    return fail(error, error_capacity, S3D_INTERNAL_ERROR, "device status 0x%x", st[0]);
}
}  // namespace s3dsp

extern "C" S3DSP_API s3d_status s3dsp_context_check(s3dsp_context* ctx, char* error,
                                                    uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "ctx is NULL");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    S3DSP_CUDA(pipe_join(ctx), "join copy streams");  // the wait then covers the copy streams too
    return check_status(ctx, error, error_capacity);
}

extern "C" S3DSP_API s3d_status s3dsp_memory_stats(int32_t device, uint64_t* reserved, uint64_t* used,
                                                  uint64_t* used_high, int32_t reset_high, char* error,
                                                  uint64_t error_capacity) {
    clear_error(error, error_capacity);
    int count = 0;
    S3DSP_CUDA(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
    if (device < 0 || device >= count || device >= 64)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "device %d out of range [0,%d)", device, count);
    cudaMemPool_t pool;
    S3DSP_CUDA(lib_pool(device, &pool), "library memory pool");
    cuuint64_t v = 0;
    if (reserved) {
        S3DSP_CUDA(cudaMemPoolGetAttribute(pool, cudaMemPoolAttrReservedMemCurrent, &v), "pool attribute");
        *reserved = v;
    }
    if (used) {
        S3DSP_CUDA(cudaMemPoolGetAttribute(pool, cudaMemPoolAttrUsedMemCurrent, &v), "pool attribute");
        *used = v;
    }
    if (used_high) {
        S3DSP_CUDA(cudaMemPoolGetAttribute(pool, cudaMemPoolAttrUsedMemHigh, &v), "pool attribute");
        *used_high = v;
    }
    if (reset_high) {
        v = 0;  // resets the high-water mark to the current use
        S3DSP_CUDA(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrUsedMemHigh, &v), "pool attribute");
    }
    return S3D_OK;
}

// ---------------------------------------------------------------------------
// Device buffers for hosts that link only this library (the counterpart of
// Backend::alloc / set_input_* / get_tensor_f32, backend.hpp:16-92)
// ---------------------------------------------------------------------------
extern "C" S3DSP_API s3d_status s3dsp_device_alloc(s3dsp_context* ctx, uint64_t bytes, void** out, char* error,
                                                  uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !out) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    *out = nullptr;
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    S3DSP_CUDA(cudaMalloc(out, bytes > 0 ? bytes : 16), "cudaMalloc");
    return S3D_OK;
}

extern "C" S3DSP_API void s3dsp_device_free(s3dsp_context* ctx, void* p) {
    if (!p) return;
    if (ctx) {
        cudaSetDevice(ctx->device);
        if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    }
    cudaFree(p);
}

extern "C" S3DSP_API s3d_status s3dsp_copy_to_device(s3dsp_context* ctx, void* d_dst, const void* h_src,
                                                    uint64_t bytes, char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || (bytes && (!d_dst || !h_src))) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    if (!bytes) return S3D_OK;
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    S3DSP_CUDA(cudaMemcpyAsync(d_dst, h_src, bytes, cudaMemcpyHostToDevice, ctx->stream), "host to device copy");
    return S3D_OK;
}

extern "C" S3DSP_API s3d_status s3dsp_copy_to_host(s3dsp_context* ctx, void* h_dst, const void* d_src, uint64_t bytes,
                                                  char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || (bytes && (!d_src || !h_dst))) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    if (bytes)
        S3DSP_CUDA(cudaMemcpyAsync(h_dst, d_src, bytes, cudaMemcpyDeviceToHost, ctx->stream), "device to host copy");
    S3DSP_CUDA(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    return S3D_OK;
}
