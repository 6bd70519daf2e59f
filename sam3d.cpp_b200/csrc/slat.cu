// SLat coarse tables (the 2x down/up-sample half of SlatTables::build,
// src/objects_runtime/sparse_ops.cpp:53-105 and :142) and the mean-pool /
// nearest-upsample gathers (slat_flow_graph.cpp:159-190), on the device.
//
// Coarse rows are the sorted unique coarse keys (b, x/2, y/2, z/2) with C++
// truncating division: the 64-bit packed key order equals lexicographic
// (b, x, y, z), so a stable radix sort of (key, fine row) pairs followed by a
// run-length pass reproduces std::map's ordering, the first-8-children rule
// and the 1/(count+1) scatter-mean quirk exactly.
#include "s3dsp_internal.h"

#include <cub/cub.cuh>

using namespace s3dsp;

struct s3dsp_slat_tables {
    int64_t nf = 0, nc = 0;
    int32_t* fine_to_coarse = nullptr;   // [nf]
    int32_t* coarse_children = nullptr;  // [8 * nc], sentinel nf
    float* coarse_inv_count = nullptr;   // [nc]
    int32_t* coarse_coords = nullptr;    // [nc, 4]
    s3dsp_hash* coarse_hash = nullptr;
    s3dsp_kmap* coarse_kmap = nullptr;   // conv_coarse
};

namespace {

__device__ __forceinline__ bool pack_key(int32_t b, int32_t x, int32_t y, int32_t z, unsigned long long& key) {
    if ((uint32_t)b > 32767u) return false;
    if (x < -32768 || x > 32767 || y < -32768 || y > 32767 || z < -32768 || z > 32767) return false;
    key = ((unsigned long long)(uint32_t)b << 48) | ((unsigned long long)(uint32_t)(x + 32768) << 32) |
          ((unsigned long long)(uint32_t)(y + 32768) << 16) | (unsigned long long)(uint32_t)(z + 32768);
    return true;
}

__global__ void coarse_key_kernel(const int4* __restrict__ coords, int64_t n, unsigned long long* __restrict__ keys,
                                  int32_t* __restrict__ rows, uint32_t* status) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int4 c = coords[i];
        unsigned long long k;
        // C++ integer division truncates toward zero (sparse_ops.cpp:63-64)
        if (!pack_key(c.x, c.y / 2, c.z / 2, c.w / 2, k)) {
            atomicOr(status, kErrCoordRange);
            k = 0;
        }
        keys[i] = k;
        rows[i] = (int32_t)i;
    }
}

// head[i] = 1 where a new coarse key starts in the sorted order
__global__ void run_head_kernel(const unsigned long long* __restrict__ skeys, int64_t n, int32_t* __restrict__ head) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        head[i] = (i == 0 || skeys[i] != skeys[i - 1]) ? 1 : 0;
}

// rank = inclusive scan of head - 1; record run starts and coarse coords
__global__ void run_scatter_kernel(const unsigned long long* __restrict__ skeys, const int32_t* __restrict__ srows,
                                   const int32_t* __restrict__ head, const int32_t* __restrict__ incl, int64_t n,
                                   int32_t* __restrict__ run_start, int4* __restrict__ ccoords,
                                   int32_t* __restrict__ f2c) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int32_t c = incl[i] - 1;
        f2c[srows[i]] = c;
        if (head[i]) {
            run_start[c] = (int32_t)i;
            const unsigned long long k = skeys[i];
            ccoords[c] = make_int4((int32_t)(k >> 48), (int32_t)((k >> 32) & 0xffff) - 32768,
                                   (int32_t)((k >> 16) & 0xffff) - 32768, (int32_t)(k & 0xffff) - 32768);
        }
    }
}

// children (first 8 fine rows of each run, ascending: the radix sort is
// stable and rows entered in ascending order) and 1/(count+1)
__global__ void children_kernel(const int32_t* __restrict__ srows, const int32_t* __restrict__ run_start, int64_t nc,
                                int64_t nf, int32_t* __restrict__ children, float* __restrict__ inv) {
    pdl_wait();
    pdl_trigger();
    for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < nc; c += (int64_t)gridDim.x * blockDim.x) {
        const int32_t b = run_start[c];
        const int32_t e = c + 1 < nc ? run_start[c + 1] : (int32_t)nf;
        const int32_t cnt = e - b;
        for (int j = 0; j < 8; ++j) children[c * 8 + j] = j < cnt ? srows[b + j] : (int32_t)nf;
        // torch scatter_reduce "mean" also counts the initial zero (sparse_ops.cpp:93-96)
        inv[c] = 1.0f / (float)(cnt + 1);
    }
}

__device__ __forceinline__ float ldf(const void* p, uint32_t dt, int64_t i) {
    if (dt == S3DSP_F32) return reinterpret_cast<const float*>(p)[i];
    if (dt == S3DSP_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    return __half2float(reinterpret_cast<const __half*>(p)[i]);
}
__device__ __forceinline__ void stf(void* p, uint32_t dt, int64_t i, float v) {
    if (dt == S3DSP_F32)
        reinterpret_cast<float*>(p)[i] = v;
    else if (dt == S3DSP_BF16)
        reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16(v);
    else
        reinterpret_cast<__half*>(p)[i] = __float2half(v);
}

// out[c] = (x[ch0] + x[ch1] + ... + x[ch7]) * inv[c], in slot order
// (slat_flow_graph.cpp:159-183); sentinel slots read zeros
__global__ void downsample_kernel(const void* __restrict__ x, uint32_t xd, int64_t nf, int c, const int32_t* __restrict__ ch,
                                  const float* __restrict__ inv, int64_t nc, void* __restrict__ y, uint32_t yd) {
    pdl_wait();
    pdl_trigger();
    const int64_t total = nc * c;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / c;
        const int k = (int)(i - r * c);
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int32_t f = ch[r * 8 + j];
            const float v = (f >= 0 && f < nf) ? ldf(x, xd, (int64_t)f * c + k) : 0.0f;
            s = j == 0 ? v : s + v;
        }
        stf(y, yd, i, s * inv[r]);
    }
}

// out[i] = x[f2c[i]] (slat_flow_graph.cpp:186-190)
__global__ void upsample_kernel(const void* __restrict__ x, uint32_t xd, int64_t nc, int c, const int32_t* __restrict__ f2c,
                                int64_t nf, void* __restrict__ y, uint32_t yd) {
    pdl_wait();
    pdl_trigger();
    const int64_t total = nf * c;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / c;
        const int k = (int)(i - r * c);
        const int32_t src = f2c[r];
        stf(y, yd, i, (src >= 0 && src < nc) ? ldf(x, xd, (int64_t)src * c + k) : 0.0f);
    }
}

inline int grid_for(int64_t n, int threads, int sm_count) {
    int64_t g = (n + threads - 1) / threads;
    const int64_t cap = (int64_t)sm_count * 16;
    if (g > cap) g = cap;
    return (int)(g < 1 ? 1 : g);
}

}  // namespace

extern "C" S3DSP_API void s3dsp_slat_tables_free(s3dsp_context* ctx, s3dsp_slat_tables* t) {
    if (!t) return;
    cudaStream_t st = ctx ? ctx->stream : nullptr;
    if (t->fine_to_coarse) cudaFreeAsync(t->fine_to_coarse, st);
    if (t->coarse_children) cudaFreeAsync(t->coarse_children, st);
    if (t->coarse_inv_count) cudaFreeAsync(t->coarse_inv_count, st);
    if (t->coarse_coords) cudaFreeAsync(t->coarse_coords, st);
    if (t->coarse_kmap) s3dsp_kmap_free(ctx, t->coarse_kmap);
    if (t->coarse_hash) s3dsp_hash_free(ctx, t->coarse_hash);
    delete t;
}

extern "C" S3DSP_API s3d_status s3dsp_slat_tables_build(s3dsp_context* ctx, const s3dsp_hash* fine,
                                                        s3dsp_slat_tables** out, char* error,
                                                        uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !fine || !out) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    *out = nullptr;
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    const int64_t n = fine->n;
    cudaStream_t st = ctx->stream;
    auto* t = new (std::nothrow) s3dsp_slat_tables();
    if (!t) return fail(error, error_capacity, S3D_OUT_OF_MEMORY, "tables allocation");
    t->nf = n;
    unsigned long long *keys = nullptr, *skeys = nullptr;
    int32_t *rows = nullptr, *srows = nullptr, *head = nullptr, *incl = nullptr, *run_start = nullptr;
    void* temp = nullptr;
    size_t temp_sort = 0, temp_scan = 0;
    cudaError_t e = cub::DeviceRadixSort::SortPairs(nullptr, temp_sort, keys, skeys, rows, srows, (int)n, 0, 64, st);
    if (e == cudaSuccess) e = cub::DeviceScan::InclusiveSum(nullptr, temp_scan, head, incl, (int)n, st);
    const size_t temp_bytes = temp_sort > temp_scan ? temp_sort : temp_scan;
    if (e == cudaSuccess) e = s3dsp::malloc_async(&keys, (size_t)n * 8, st);
    if (e == cudaSuccess) e = s3dsp::malloc_async(&skeys, (size_t)n * 8, st);
    if (e == cudaSuccess) e = s3dsp::malloc_async(&rows, (size_t)n * 4, st);
    if (e == cudaSuccess) e = s3dsp::malloc_async(&srows, (size_t)n * 4, st);
    if (e == cudaSuccess) e = s3dsp::malloc_async(&head, (size_t)n * 4, st);
    if (e == cudaSuccess) e = s3dsp::malloc_async(&incl, (size_t)n * 4, st);
    if (e == cudaSuccess) e = s3dsp::malloc_async(&run_start, (size_t)n * 4, st);
    if (e == cudaSuccess) e = s3dsp::malloc_async(&temp, temp_bytes > 0 ? temp_bytes : 16, st);
    if (e == cudaSuccess) e = s3dsp::malloc_async(&t->fine_to_coarse, (size_t)n * 4, st);
    if (e == cudaSuccess) e = s3dsp::malloc_async(&t->coarse_coords, (size_t)n * 16, st);  // nc <= nf
    s3d_status status = S3D_OK;
    int32_t nc = 0;
    if (e == cudaSuccess) {
        const int g = grid_for(n, 256, ctx->sm_count);
        launch_pdl(coarse_key_kernel, dim3(g), dim3(256), 0, st, reinterpret_cast<const int4*>(fine->coords), n, keys,
                   rows, ctx->d_status);
        size_t tb = temp_bytes;
        e = cub::DeviceRadixSort::SortPairs(temp, tb, keys, skeys, rows, srows, (int)n, 0, 64, st);
        if (e == cudaSuccess) {
            launch_pdl(run_head_kernel, dim3(g), dim3(256), 0, st, skeys, n, head);
            tb = temp_bytes;
            e = cub::DeviceScan::InclusiveSum(temp, tb, head, incl, (int)n, st);
        }
        if (e == cudaSuccess) {
            launch_pdl(run_scatter_kernel, dim3(g), dim3(256), 0, st, skeys, srows, head, incl, n, run_start,
                                                  reinterpret_cast<int4*>(t->coarse_coords), t->fine_to_coarse);
            e = cudaMemcpyAsync(&nc, incl + (n - 1), 4, cudaMemcpyDeviceToHost, st);
        }
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e == cudaSuccess) {
            t->nc = nc;
            status = check_status(ctx, error, error_capacity);
        }
    }
    if (e == cudaSuccess && status == S3D_OK) {
        e = s3dsp::malloc_async(&t->coarse_children, (size_t)nc * 8 * 4, st);
        if (e == cudaSuccess) e = s3dsp::malloc_async(&t->coarse_inv_count, (size_t)nc * 4, st);
        if (e == cudaSuccess) {
            launch_pdl(children_kernel, dim3(grid_for(nc, 256, ctx->sm_count)), dim3(256), 0, st, srows, run_start,
                       nc, n, t->coarse_children, t->coarse_inv_count);
            e = cudaGetLastError();
        }
    }
    for (void* pz : {(void*)keys, (void*)skeys, (void*)rows, (void*)srows, (void*)head, (void*)incl,
                     (void*)run_start, temp})
        if (pz) cudaFreeAsync(pz, st);
    if (e != cudaSuccess) status = cuda_fail(error, error_capacity, e, "slat coarse tables");
    if (status == S3D_OK) {
        // conv_coarse: submanifold map of the coarse set (sparse_ops.cpp:142)
        status = s3dsp_hash_build(ctx, t->coarse_coords, nc, 0, &t->coarse_hash, error, error_capacity);
        if (status == S3D_OK) status = s3dsp_kmap_build_subm3(ctx, t->coarse_hash, &t->coarse_kmap, error, error_capacity);
    }
    if (status != S3D_OK) {
        s3dsp_slat_tables_free(ctx, t);
        return status;
    }
    *out = t;
    return S3D_OK;
}

extern "C" S3DSP_API int64_t s3dsp_slat_tables_coarse_rows(const s3dsp_slat_tables* t) { return t ? t->nc : 0; }

extern "C" S3DSP_API const s3dsp_kmap* s3dsp_slat_tables_coarse_kmap(const s3dsp_slat_tables* t) {
    return t ? t->coarse_kmap : nullptr;
}

extern "C" S3DSP_API s3d_status s3dsp_slat_tables_export(s3dsp_context* ctx, const s3dsp_slat_tables* t,
                                                         int32_t* d_fine_to_coarse, int32_t* d_coarse_children,
                                                         float* d_coarse_inv_count, int32_t* d_coarse_coords,
                                                         char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !t) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    cudaStream_t st = ctx->stream;
    if (d_fine_to_coarse)
        S3DSP_CUDA(cudaMemcpyAsync(d_fine_to_coarse, t->fine_to_coarse, (size_t)t->nf * 4, cudaMemcpyDeviceToDevice, st), "copy");
    if (d_coarse_children)
        S3DSP_CUDA(cudaMemcpyAsync(d_coarse_children, t->coarse_children, (size_t)t->nc * 32, cudaMemcpyDeviceToDevice, st), "copy");
    if (d_coarse_inv_count)
        S3DSP_CUDA(cudaMemcpyAsync(d_coarse_inv_count, t->coarse_inv_count, (size_t)t->nc * 4, cudaMemcpyDeviceToDevice, st), "copy");
    if (d_coarse_coords)
        S3DSP_CUDA(cudaMemcpyAsync(d_coarse_coords, t->coarse_coords, (size_t)t->nc * 16, cudaMemcpyDeviceToDevice, st), "copy");
    return S3D_OK;
}

extern "C" S3DSP_API s3d_status s3dsp_slat_downsample(s3dsp_context* ctx, const s3dsp_slat_tables* t, const void* x,
                                                      uint32_t x_dtype, int64_t c, void* y, uint32_t y_dtype,
                                                      char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !t || !x || !y) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    if (!dtype_ok(x_dtype) || !dtype_ok(y_dtype) || c <= 0) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "bad dtype/channels");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    launch_pdl(downsample_kernel, dim3(grid_for(t->nc * c, 256, ctx->sm_count)), dim3(256), 0, ctx->stream, x,
               x_dtype, t->nf, (int)c, t->coarse_children, t->coarse_inv_count, t->nc, y, y_dtype);
    S3DSP_LAUNCH_CHECK("downsample_kernel");
    return S3D_OK;
}

extern "C" S3DSP_API s3d_status s3dsp_slat_upsample(s3dsp_context* ctx, const s3dsp_slat_tables* t, const void* x,
                                                    uint32_t x_dtype, int64_t c, void* y, uint32_t y_dtype,
                                                    char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !t || !x || !y) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    if (!dtype_ok(x_dtype) || !dtype_ok(y_dtype) || c <= 0) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "bad dtype/channels");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    launch_pdl(upsample_kernel, dim3(grid_for(t->nf * c, 256, ctx->sm_count)), dim3(256), 0, ctx->stream, x, x_dtype,
               t->nc, (int)c, t->fine_to_coarse, t->nf, y, y_dtype);
    S3DSP_LAUNCH_CHECK("upsample_kernel");
    return S3D_OK;
}
