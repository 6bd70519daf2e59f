// The coordinate pipeline in front of the sparse path, on the device:
//   * SS occupancy argwhere           src/objects_runtime/session.cpp:1436-1441
//   * prune_surface_coords            src/objects_runtime/session.cpp:129-166
//   * downsample_coords               src/objects_runtime/session.cpp:168-236
// All three keep their input order (flags -> exclusive scan -> scatter).
// Neighbour membership and "first occurrence" use the coordinate hash
// (first row of a key = its first insertion, as std::unordered_set::insert
// keeps the first). The downsample mapping uses double arithmetic with
// explicitly rounded, unfused operations, as the reference is built
// (-ffp-contract=off); its rare random subsample (std::shuffle with
// std::mt19937) runs on the host, as in the reference. Each call returns the
// row count to the host, so it synchronises the context's stream.
#include "hash_view.cuh"
#include "s3dsp_internal.h"

#include <cub/cub.cuh>

#include <algorithm>
#include <cmath>
#include <numeric>
#include <random>
#include <vector>

using namespace s3dsp;
using namespace s3dsp::hash;

namespace {

inline int grid_for(int64_t n, int threads, int sm_count) {
    int64_t g = (n + threads - 1) / threads;
    const int64_t cap = (int64_t)sm_count * 16;
    if (g > cap) g = cap;
    return (int)(g < 1 ? 1 : g);
}

__global__ void occ_flag_kernel(const float* __restrict__ occ, int64_t total, int32_t* __restrict__ flag) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x)
        flag[i] = occ[i] > 0.0f ? 1 : 0;
}

__global__ void occ_scatter_kernel(const int32_t* __restrict__ flag, const int32_t* __restrict__ pos, int64_t total,
                                   int32_t ny, int32_t nz, int32_t batch, int4* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x)
        if (flag[i]) {
            const int32_t z = (int32_t)(i % nz);
            const int64_t xy = i / nz;
            out[pos[i]] = make_int4(batch, (int32_t)(xy / ny), (int32_t)(xy % ny), z);
        }
}

// surface: some cell of the (2d+1)^3 neighbourhood is not in the set
__global__ void prune_flag_kernel(const int4* __restrict__ coords, int64_t n, HashView h, int32_t d,
                                  int32_t* __restrict__ flag) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int4 c = coords[i];
        int32_t surface = 0;
        for (int dx = -d; dx <= d && !surface; ++dx)
            for (int dy = -d; dy <= d && !surface; ++dy)
                for (int dz = -d; dz <= d && !surface; ++dz)
                    surface = h.find_coord(c.x, c.y + dx, c.z + dy, c.w + dz) < 0;
        flag[i] = surface;
    }
}

__global__ void select_scatter_kernel(const int4* __restrict__ in, const int32_t* __restrict__ flag,
                                      const int32_t* __restrict__ pos, int64_t n, int4* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        if (flag[i]) out[pos[i]] = in[i];
}

__global__ void bounds_kernel(const int4* __restrict__ coords, int64_t n, int32_t* __restrict__ lohi) {
    pdl_wait();
    pdl_trigger();
    int32_t lo[3] = {INT32_MAX, INT32_MAX, INT32_MAX}, hi[3] = {INT32_MIN, INT32_MIN, INT32_MIN};
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int4 c = coords[i];
        lo[0] = min(lo[0], c.y), lo[1] = min(lo[1], c.z), lo[2] = min(lo[2], c.w);
        hi[0] = max(hi[0], c.y), hi[1] = max(hi[1], c.z), hi[2] = max(hi[2], c.w);
    }
    for (int c = 0; c < 3; ++c) {
        atomicMin(lohi + c, lo[c]);
        atomicMax(lohi + 3 + c, hi[c]);
    }
}

struct DownsampleAxes {
    int32_t lo[3];
    double denom[3];    // hi - lo
    double tm1[3];      // target - 1
    double tmin[3];     // target min (double)
    int32_t tmin_i[3];  // target min, truncated
    int32_t tmax_i[3];  // target max, truncated
};

// the reference's per-axis rescale, with every double operation rounded
// separately (no fused multiply-add)
__global__ void downsample_map_kernel(const int4* __restrict__ coords, int64_t n, DownsampleAxes ax,
                                      int4* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int4 c = coords[i];
        const int32_t v[3] = {c.y, c.z, c.w};
        int32_t o[3];
#pragma unroll
        for (int a = 0; a < 3; ++a) {
            const double normalized =
                ax.denom[a] > 0.0 ? __ddiv_rn(__dsub_rn((double)v[a], (double)ax.lo[a]), ax.denom[a]) : 0.0;
            const double value = __dadd_rn(__dmul_rn(normalized, ax.tm1[a]), ax.tmin[a]);
            int64_t r = (int64_t)floor(__dadd_rn(value, 0.5));
            r = max(r, (int64_t)ax.tmin_i[a]);
            r = min(r, (int64_t)ax.tmax_i[a]);
            o[a] = (int32_t)r;
        }
        out[i] = make_int4(c.x, o[0], o[1], o[2]);
    }
}

// first occurrence of each coordinate: the row the hash kept for its key
__global__ void first_flag_kernel(const int4* __restrict__ coords, int64_t n, HashView h, int32_t* __restrict__ flag) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int4 c = coords[i];
        flag[i] = h.find_coord(c.x, c.y, c.z, c.w) == (int32_t)i;
    }
}

// Device scratch of one call, released on the stream at scope exit.
struct Scratch {
    cudaStream_t s;
    std::vector<void*> ptrs;
    explicit Scratch(cudaStream_t st) : s(st) {}
    ~Scratch() {
        for (void* p : ptrs) cudaFreeAsync(p, s);
    }
    template <typename T>
    cudaError_t get(T** p, size_t bytes) {
        void* q = nullptr;
        const cudaError_t e = s3dsp::malloc_async(&q, bytes > 0 ? bytes : 16, s);
        if (e == cudaSuccess) ptrs.push_back(q);
        *p = static_cast<T*>(q);
        return e;
    }
};

// flags -> exclusive positions and the selected count (host; synchronises)
cudaError_t scan_flags(s3dsp_context* ctx, Scratch& sc, const int32_t* flag, int64_t n, int32_t** pos,
                       int64_t* count) {
    cudaStream_t st = ctx->stream;
    size_t tb = 0;
    cudaError_t e = cub::DeviceScan::ExclusiveSum(nullptr, tb, flag, (int32_t*)nullptr, (int)n, st);
    void* temp = nullptr;
    if (e == cudaSuccess) e = sc.get(&temp, tb);
    if (e == cudaSuccess) e = sc.get(pos, sizeof(int32_t) * (size_t)n);
    if (e == cudaSuccess) e = cub::DeviceScan::ExclusiveSum(temp, tb, flag, *pos, (int)n, st);
    int32_t last[2] = {0, 0};
    if (e == cudaSuccess) e = cudaMemcpyAsync(&last[0], *pos + (n - 1), 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(&last[1], flag + (n - 1), 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    *count = (int64_t)last[0] + last[1];
    return e;
}

}  // namespace

extern "C" S3DSP_API s3d_status s3dsp_occupancy_coords(s3dsp_context* ctx, const float* d_occ, int32_t nx, int32_t ny,
                                                       int32_t nz, int32_t batch, int32_t* d_coords, int64_t capacity,
                                                       int64_t* count, char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !d_occ || !count) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    *count = 0;
    const int64_t total = (int64_t)nx * ny * nz;
    if (nx <= 0 || ny <= 0 || nz <= 0 || total >= (1ll << 31))
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "grid %d x %d x %d", nx, ny, nz);
    if (capacity > 0 && (!d_coords || ((uintptr_t)d_coords & 15)))
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "d_coords must be a 16-byte aligned device pointer");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    cudaStream_t st = ctx->stream;
    Scratch sc(st);
    int32_t *flag, *pos;
    S3DSP_CUDA(sc.get(&flag, sizeof(int32_t) * (size_t)total), "scratch");
    launch_pdl(occ_flag_kernel, dim3(grid_for(total, 256, ctx->sm_count)), dim3(256), 0, st, d_occ, total, flag);
    S3DSP_LAUNCH_CHECK("occ_flag_kernel");
    int64_t n = 0;
    S3DSP_CUDA(scan_flags(ctx, sc, flag, total, &pos, &n), "occupancy scan");
    *count = n;
    if (n > capacity)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "%lld occupied cells > capacity %lld", (long long)n,
                    (long long)capacity);
    launch_pdl(occ_scatter_kernel, dim3(grid_for(total, 256, ctx->sm_count)), dim3(256), 0, st, flag, pos, total, ny,
               nz, batch, reinterpret_cast<int4*>(d_coords));
    S3DSP_LAUNCH_CHECK("occ_scatter_kernel");
    return S3D_OK;
}

extern "C" S3DSP_API s3d_status s3dsp_prune_surface(s3dsp_context* ctx, const int32_t* d_coords, int64_t n,
                                                    int32_t max_axis_dist, int32_t* d_out, int64_t capacity,
                                                    int64_t* count, char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !d_coords || !count) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    *count = 0;
    if (n <= 0) return n == 0 ? S3D_OK : fail(error, error_capacity, S3D_INVALID_ARGUMENT, "negative count");
    if (max_axis_dist < 1 || max_axis_dist > 8)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "max_axis_dist %d outside 1..8", max_axis_dist);
    if (!d_out || ((uintptr_t)d_out & 15))
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "d_out must be a 16-byte aligned device pointer");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    s3dsp_hash* h = nullptr;
    S3DSP_TRY(s3dsp_hash_build(ctx, d_coords, n, 0, &h, error, error_capacity));
    cudaStream_t st = ctx->stream;
    s3d_status status = S3D_OK;
    {
        Scratch sc(st);
        int32_t *flag = nullptr, *pos = nullptr;
        cudaError_t e = sc.get(&flag, sizeof(int32_t) * (size_t)n);
        if (e == cudaSuccess) {
            launch_pdl(prune_flag_kernel, dim3(grid_for(n, 256, ctx->sm_count)), dim3(256), 0, st,
                       reinterpret_cast<const int4*>(h->coords), n, view_of(h), max_axis_dist, flag);
            e = cudaGetLastError();
        }
        int64_t m = 0;
        if (e == cudaSuccess) e = scan_flags(ctx, sc, flag, n, &pos, &m);
        if (e != cudaSuccess) {
            status = cuda_fail(error, error_capacity, e, "prune_surface");
        } else {
            *count = m;
            if (m > capacity) {
                status = fail(error, error_capacity, S3D_INVALID_ARGUMENT, "%lld surface rows > capacity %lld",
                              (long long)m, (long long)capacity);
            } else {
                launch_pdl(select_scatter_kernel, dim3(grid_for(n, 256, ctx->sm_count)), dim3(256), 0, st,
                           reinterpret_cast<const int4*>(h->coords), flag, pos, n, reinterpret_cast<int4*>(d_out));
                e = cudaGetLastError();
                if (e != cudaSuccess) status = cuda_fail(error, error_capacity, e, "select_scatter_kernel");
            }
        }
    }
    s3dsp_hash_free(ctx, h);
    return status;
}

extern "C" S3DSP_API s3d_status s3dsp_downsample_coords(s3dsp_context* ctx, const int32_t* d_coords, int64_t n,
                                                        int64_t max_coords, int32_t factor, uint32_t seed,
                                                        int32_t* d_out, int64_t capacity, int64_t* count, char* error,
                                                        uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !d_coords || !count) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    *count = 0;
    if (n < 0 || max_coords < 0 || factor <= 0)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "bad n / max_coords / factor");
    if (n == 0) return S3D_OK;
    if (!d_out || ((uintptr_t)d_out & 15) || ((uintptr_t)d_coords & 15))
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "coordinates must be 16-byte aligned device pointers");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    cudaStream_t st = ctx->stream;
    if (n <= max_coords) {  // the reference returns its input unchanged
        if (n > capacity)
            return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "%lld rows > capacity %lld", (long long)n,
                        (long long)capacity);
        S3DSP_CUDA(cudaMemcpyAsync(d_out, d_coords, (size_t)n * 16, cudaMemcpyDeviceToDevice, st), "copy");
        S3DSP_CUDA(cudaStreamSynchronize(st), "cudaStreamSynchronize");
        *count = n;
        return S3D_OK;
    }
    // per-axis bounds
    Scratch sc(st);
    int32_t* lohi;
    S3DSP_CUDA(sc.get(&lohi, 6 * sizeof(int32_t)), "scratch");
    const int32_t init[6] = {INT32_MAX, INT32_MAX, INT32_MAX, INT32_MIN, INT32_MIN, INT32_MIN};
    S3DSP_CUDA(cudaMemcpyAsync(lohi, init, sizeof init, cudaMemcpyHostToDevice, st), "bounds init");
    launch_pdl(bounds_kernel, dim3(grid_for(n, 256, ctx->sm_count)), dim3(256), 0, st,
               reinterpret_cast<const int4*>(d_coords), n, lohi);
    S3DSP_LAUNCH_CHECK("bounds_kernel");
    int32_t hb[6];
    S3DSP_CUDA(cudaMemcpyAsync(hb, lohi, sizeof hb, cudaMemcpyDeviceToHost, st), "bounds");
    S3DSP_CUDA(cudaStreamSynchronize(st), "cudaStreamSynchronize");
    // the reference's per-axis targets, in the same double expressions
    DownsampleAxes ax;
    for (int c = 0; c < 3; ++c) {
        const int32_t lo = hb[c], hi = hb[3 + c];
        const double original = (double)(hi - lo + 1);
        const double target = original / (double)factor;
        volatile double offset = (original - target) * 0.5;  // volatile: no fused multiply-add
        const double tmin = (double)lo + offset;
        const double tmax = tmin + target - 1.0;
        ax.lo[c] = lo;
        ax.denom[c] = (double)(hi - lo);
        ax.tm1[c] = target - 1.0;
        ax.tmin[c] = tmin;
        ax.tmin_i[c] = (int32_t)tmin;  // truncation toward zero, as torch .int()
        ax.tmax_i[c] = (int32_t)tmax;
    }
    int32_t* mapped;
    S3DSP_CUDA(sc.get(&mapped, (size_t)n * 16), "scratch");
    launch_pdl(downsample_map_kernel, dim3(grid_for(n, 256, ctx->sm_count)), dim3(256), 0, st,
               reinterpret_cast<const int4*>(d_coords), n, ax, reinterpret_cast<int4*>(mapped));
    S3DSP_LAUNCH_CHECK("downsample_map_kernel");
    // first occurrences, in input order
    s3dsp_hash* h = nullptr;
    S3DSP_TRY(s3dsp_hash_build(ctx, mapped, n, 0, &h, error, error_capacity));
    int32_t *flag = nullptr, *pos = nullptr, *uniq = nullptr;
    cudaError_t e = sc.get(&flag, sizeof(int32_t) * (size_t)n);
    if (e == cudaSuccess) {
        launch_pdl(first_flag_kernel, dim3(grid_for(n, 256, ctx->sm_count)), dim3(256), 0, st,
                   reinterpret_cast<const int4*>(mapped), n, view_of(h), flag);
        e = cudaGetLastError();
    }
    int64_t un = 0;
    if (e == cudaSuccess) e = scan_flags(ctx, sc, flag, n, &pos, &un);
    if (e == cudaSuccess) e = sc.get(&uniq, (size_t)un * 16);
    if (e == cudaSuccess) {
        launch_pdl(select_scatter_kernel, dim3(grid_for(n, 256, ctx->sm_count)), dim3(256), 0, st,
                   reinterpret_cast<const int4*>(mapped), flag, pos, n, reinterpret_cast<int4*>(uniq));
        e = cudaGetLastError();
    }
    s3dsp_hash_free(ctx, h);
    if (e != cudaSuccess) return cuda_fail(error, error_capacity, e, "downsample_coords");
    const int64_t m = un > max_coords ? max_coords : un;
    *count = m;
    if (m > capacity)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "%lld rows > capacity %lld", (long long)m,
                    (long long)capacity);
    if (un <= max_coords) {
        S3DSP_CUDA(cudaMemcpyAsync(d_out, uniq, (size_t)un * 16, cudaMemcpyDeviceToDevice, st), "copy");
        S3DSP_CUDA(cudaStreamSynchronize(st), "cudaStreamSynchronize");
        return S3D_OK;
    }
    // more unique rows than allowed: the reference's seeded random subsample, on the host
    std::vector<int32_t> hu((size_t)un * 4), hs((size_t)max_coords * 4);
    S3DSP_CUDA(cudaMemcpyAsync(hu.data(), uniq, (size_t)un * 16, cudaMemcpyDeviceToHost, st), "D2H");
    S3DSP_CUDA(cudaStreamSynchronize(st), "cudaStreamSynchronize");
    std::mt19937 rng(seed);
    std::vector<size_t> order((size_t)un);
    std::iota(order.begin(), order.end(), 0);
    std::shuffle(order.begin(), order.end(), rng);
    for (int64_t j = 0; j < max_coords; ++j)
        std::copy_n(&hu[order[(size_t)j] * 4], 4, &hs[(size_t)j * 4]);
    S3DSP_CUDA(cudaMemcpyAsync(d_out, hs.data(), (size_t)max_coords * 16, cudaMemcpyHostToDevice, st), "H2D");
    S3DSP_CUDA(cudaStreamSynchronize(st), "cudaStreamSynchronize");
    return S3D_OK;
}
