// GS decoder Swin window tables and absolute position embedding on the
// device: GsTables::build (src/objects_runtime/sparse_ops.cpp:182-270).
//
// A token's window is (b, (x+s)/W, (y+s)/W, (z+s)/W) with C division; a
// window's id is the order of its first token (the reference's map assigns
// ids as windows are first met). Here: the coordinate hash over window keys
// keeps each key's first row (atomicMin), so "is the first row of its
// window" is one probe, and the window ids are an exclusive scan of those
// flags. Tokens are grouped by a stable radix sort on window id (table order
// inside a window), windows are ordered by a stable radix sort on token count
// (id order inside a count), and a scan of the counts in that order gives
// every window's first bucket row. The bucket list (one entry per distinct
// count, a few dozen) is finished on the host.
#include "hash_view.cuh"
#include "s3dsp_internal.h"

#include <cub/cub.cuh>

#include <cmath>
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

#define GRID_LOOP(i, n) \
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (n); i += (int64_t)gridDim.x * blockDim.x)

__global__ void window_key_kernel(const int4* __restrict__ coords, int64_t n, int32_t shift, int32_t window,
                                  int4* __restrict__ wc) {
    pdl_wait();
    pdl_trigger();
    GRID_LOOP(i, n) {
        const int4 c = coords[i];
        wc[i] = make_int4(c.x, (c.y + shift) / window, (c.z + shift) / window, (c.w + shift) / window);
    }
}

__global__ void first_of_window_kernel(const int4* __restrict__ wc, int64_t n, HashView h, int32_t* __restrict__ fr,
                                       int32_t* __restrict__ is_first) {
    pdl_wait();
    pdl_trigger();
    GRID_LOOP(i, n) {
        const int4 k = wc[i];
        const int32_t f = h.find_coord(k.x, k.y, k.z, k.w);
        fr[i] = f;
        is_first[i] = f == (int32_t)i;
    }
}

__global__ void window_id_kernel(const int32_t* __restrict__ fr, const int32_t* __restrict__ first_rank, int64_t n,
                                 int32_t* __restrict__ wid, int32_t* __restrict__ rows, int32_t* __restrict__ cnt) {
    pdl_wait();
    pdl_trigger();
    GRID_LOOP(i, n) {
        const int32_t w = first_rank[fr[i]];
        wid[i] = w;
        rows[i] = (int32_t)i;
        atomicAdd(cnt + w, 1);
    }
}

__global__ void iota_kernel(int32_t* __restrict__ v, int64_t n) {
    pdl_wait();
    pdl_trigger();
    GRID_LOOP(i, n) v[i] = (int32_t)i;
}

__global__ void window_offset_scatter_kernel(const int32_t* __restrict__ win_by_len,
                                             const int32_t* __restrict__ off_by_len, int64_t nw,
                                             int32_t* __restrict__ win_off) {
    pdl_wait();
    pdl_trigger();
    GRID_LOOP(k, nw) win_off[win_by_len[k]] = off_by_len[k];
}

__global__ void bucket_rows_kernel(const int32_t* __restrict__ swid, const int32_t* __restrict__ srow, int64_t n,
                                   const int32_t* __restrict__ seg_start, const int32_t* __restrict__ win_off,
                                   int32_t* __restrict__ bkt_idx, int32_t* __restrict__ bwd_idx) {
    pdl_wait();
    pdl_trigger();
    GRID_LOOP(p, n) {
        const int32_t w = swid[p], r = srow[p];
        const int32_t out = win_off[w] + ((int32_t)p - seg_start[w]);
        bkt_idx[out] = r;
        bwd_idx[r] = out;
    }
}

__global__ void ape_kernel(const int4* __restrict__ coords, int64_t n, int32_t f, const float* __restrict__ freq,
                           float* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const int64_t total = n * 3 * f;
    GRID_LOOP(j, total) {
        const int32_t i = (int32_t)(j % f);
        const int64_t ta = j / f;
        const int32_t a = (int32_t)(ta % 3);
        const int64_t t = ta / 3;
        const int4 c = coords[t];
        const float v = (float)(a == 0 ? c.y : a == 1 ? c.z : c.w);
        const float ph = v * freq[i];
        float* o = out + t * (int64_t)(6 * f) + (int64_t)a * 2 * f;
        o[i] = sinf(ph);
        o[f + i] = cosf(ph);
    }
}

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

int bits_for(int64_t v) {
    int b = 1;
    while (b < 31 && ((int64_t)1 << b) <= v) ++b;
    return b;
}

}  // namespace

extern "C" S3DSP_API s3d_status s3dsp_gs_window_tables(s3dsp_context* ctx, const int32_t* d_coords, int64_t n,
                                                       int32_t shift, int32_t window, int32_t* d_bkt_idx,
                                                       int32_t* d_bwd_idx, int32_t* h_buckets,
                                                       int64_t bucket_capacity, int64_t* n_buckets, char* error,
                                                       uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !d_coords || !d_bkt_idx || !d_bwd_idx || !n_buckets)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    *n_buckets = 0;
    if (n <= 0 || n >= (1ll << 31)) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "token count %lld", (long long)n);
    if (window <= 0 || shift < 0) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "window %d / shift %d", window, shift);
    if ((uintptr_t)d_coords & 15)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "d_coords must be 16-byte aligned");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    cudaStream_t st = ctx->stream;
    const int g = grid_for(n, 256, ctx->sm_count);
    Scratch sc(st);
    int32_t* wc;
    S3DSP_CUDA(sc.get(&wc, (size_t)n * 16), "scratch");
    launch_pdl(window_key_kernel, dim3(g), dim3(256), 0, st, reinterpret_cast<const int4*>(d_coords), n, shift, window,
                                         reinterpret_cast<int4*>(wc));
    S3DSP_LAUNCH_CHECK("window_key_kernel");
    s3dsp_hash* h = nullptr;
    S3DSP_TRY(s3dsp_hash_build(ctx, wc, n, 0, &h, error, error_capacity));
    int32_t *fr, *is_first, *rank, *wid, *rows, *swid, *srow;
    cudaError_t e = sc.get(&fr, 4 * (size_t)n);
    if (e == cudaSuccess) e = sc.get(&is_first, 4 * (size_t)n);
    if (e == cudaSuccess) e = sc.get(&rank, 4 * (size_t)n);
    if (e == cudaSuccess) e = sc.get(&wid, 4 * (size_t)n);
    if (e == cudaSuccess) e = sc.get(&rows, 4 * (size_t)n);
    if (e == cudaSuccess) e = sc.get(&swid, 4 * (size_t)n);
    if (e == cudaSuccess) e = sc.get(&srow, 4 * (size_t)n);
    if (e == cudaSuccess) {
        launch_pdl(first_of_window_kernel, dim3(g), dim3(256), 0, st, reinterpret_cast<const int4*>(wc), n,
                   view_of(h), fr, is_first);
        e = cudaGetLastError();
    }
    // window ids in first-appearance order
    size_t tb = 0;
    void* temp = nullptr;
    if (e == cudaSuccess) e = cub::DeviceScan::ExclusiveSum(nullptr, tb, is_first, rank, (int)n, st);
    if (e == cudaSuccess) e = sc.get(&temp, tb);
    if (e == cudaSuccess) e = cub::DeviceScan::ExclusiveSum(temp, tb, is_first, rank, (int)n, st);
    int32_t last[2] = {0, 0};
    if (e == cudaSuccess) e = cudaMemcpyAsync(&last[0], rank + (n - 1), 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(&last[1], is_first + (n - 1), 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    const int64_t nw = (int64_t)last[0] + last[1];
    int32_t *cnt = nullptr, *seg_start = nullptr, *win = nullptr, *slen = nullptr, *swin = nullptr,
            *off_by_len = nullptr, *win_off = nullptr;
    if (e == cudaSuccess) e = sc.get(&cnt, 4 * (size_t)nw);
    if (e == cudaSuccess) e = sc.get(&seg_start, 4 * (size_t)nw);
    if (e == cudaSuccess) e = sc.get(&win, 4 * (size_t)nw);
    if (e == cudaSuccess) e = sc.get(&slen, 4 * (size_t)nw);
    if (e == cudaSuccess) e = sc.get(&swin, 4 * (size_t)nw);
    if (e == cudaSuccess) e = sc.get(&off_by_len, 4 * (size_t)nw);
    if (e == cudaSuccess) e = sc.get(&win_off, 4 * (size_t)nw);
    if (e == cudaSuccess) e = cudaMemsetAsync(cnt, 0, 4 * (size_t)nw, st);
    if (e == cudaSuccess) {
        launch_pdl(window_id_kernel, dim3(g), dim3(256), 0, st, fr, rank, n, wid, rows, cnt);
        e = cudaGetLastError();
    }
    // tokens grouped by window (stable: table order inside a window)
    const int wbits = bits_for(nw);
    size_t tb2 = 0;
    void* temp2 = nullptr;
    if (e == cudaSuccess) e = cub::DeviceRadixSort::SortPairs(nullptr, tb2, wid, swid, rows, srow, (int)n, 0, wbits, st);
    if (e == cudaSuccess) e = sc.get(&temp2, tb2);
    if (e == cudaSuccess) e = cub::DeviceRadixSort::SortPairs(temp2, tb2, wid, swid, rows, srow, (int)n, 0, wbits, st);
    // window segments in id order
    size_t tb3 = 0;
    void* temp3 = nullptr;
    if (e == cudaSuccess) e = cub::DeviceScan::ExclusiveSum(nullptr, tb3, cnt, seg_start, (int)nw, st);
    if (e == cudaSuccess) e = sc.get(&temp3, tb3);
    if (e == cudaSuccess) e = cub::DeviceScan::ExclusiveSum(temp3, tb3, cnt, seg_start, (int)nw, st);
    // windows by token count (stable: id order inside a count)
    if (e == cudaSuccess) {
        launch_pdl(iota_kernel, dim3(grid_for(nw, 256, ctx->sm_count)), dim3(256), 0, st, win, nw);
        e = cudaGetLastError();
    }
    const int lbits = bits_for(n);
    size_t tb4 = 0;
    void* temp4 = nullptr;
    if (e == cudaSuccess) e = cub::DeviceRadixSort::SortPairs(nullptr, tb4, cnt, slen, win, swin, (int)nw, 0, lbits, st);
    if (e == cudaSuccess) e = sc.get(&temp4, tb4);
    if (e == cudaSuccess) e = cub::DeviceRadixSort::SortPairs(temp4, tb4, cnt, slen, win, swin, (int)nw, 0, lbits, st);
    size_t tb5 = 0;
    void* temp5 = nullptr;
    if (e == cudaSuccess) e = cub::DeviceScan::ExclusiveSum(nullptr, tb5, slen, off_by_len, (int)nw, st);
    if (e == cudaSuccess) e = sc.get(&temp5, tb5);
    if (e == cudaSuccess) e = cub::DeviceScan::ExclusiveSum(temp5, tb5, slen, off_by_len, (int)nw, st);
    if (e == cudaSuccess) {
        launch_pdl(window_offset_scatter_kernel, dim3(grid_for(nw, 256, ctx->sm_count)), dim3(256), 0, st, swin,
                   off_by_len, nw, win_off);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) {
        launch_pdl(bucket_rows_kernel, dim3(g), dim3(256), 0, st, swid, srow, n, seg_start, win_off, d_bkt_idx,
                   d_bwd_idx);
        e = cudaGetLastError();
    }
    // bucket list on the host: one entry per distinct token count
    std::vector<int32_t> hlen((size_t)nw);
    if (e == cudaSuccess) e = cudaMemcpyAsync(hlen.data(), slen, 4 * (size_t)nw, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    s3dsp_hash_free(ctx, h);
    if (e != cudaSuccess) return cuda_fail(error, error_capacity, e, "gs window tables");
    int64_t nb = 0, row = 0;
    for (int64_t k = 0; k < nw; ++k) {
        if (k == 0 || hlen[(size_t)k] != hlen[(size_t)k - 1]) {
            if (nb < bucket_capacity && h_buckets) {
                h_buckets[3 * nb + 0] = hlen[(size_t)k];
                h_buckets[3 * nb + 1] = (int32_t)row;
                h_buckets[3 * nb + 2] = 0;
            }
            ++nb;
        }
        if (nb - 1 < bucket_capacity && h_buckets) ++h_buckets[3 * (nb - 1) + 2];
        row += hlen[(size_t)k];
    }
    *n_buckets = nb;
    if (nb > bucket_capacity)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "%lld buckets > capacity %lld", (long long)nb,
                    (long long)bucket_capacity);
    return S3D_OK;
}

extern "C" S3DSP_API s3d_status s3dsp_ape(s3dsp_context* ctx, const int32_t* d_coords, int64_t n, int32_t channels,
                                          float* d_out, char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !d_coords || !d_out) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    if (n < 0 || channels <= 0 || channels % 6)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "channels %d must be a positive multiple of 6", channels);
    if (n == 0) return S3D_OK;
    if ((uintptr_t)d_coords & 15) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "d_coords must be 16-byte aligned");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    const int32_t f = channels / 6;
    // frequencies with the host's powf, as the reference computes them
    std::vector<float> freq((size_t)f);
    for (int32_t i = 0; i < f; ++i) freq[(size_t)i] = 1.0f / powf(10000.0f, (float)i / (float)f);
    cudaStream_t st = ctx->stream;
    Scratch sc(st);
    float* dfreq;
    S3DSP_CUDA(sc.get(&dfreq, 4 * (size_t)f), "scratch");
    S3DSP_CUDA(cudaMemcpyAsync(dfreq, freq.data(), 4 * (size_t)f, cudaMemcpyHostToDevice, st), "H2D");
    launch_pdl(ape_kernel, dim3(grid_for(n * 3 * f, 256, ctx->sm_count)), dim3(256), 0, st,
               reinterpret_cast<const int4*>(d_coords), n, f, dfreq, d_out);
    S3DSP_LAUNCH_CHECK("ape_kernel");
    return S3D_OK;  // a copy from pageable memory has been staged when cudaMemcpyAsync returns
}
