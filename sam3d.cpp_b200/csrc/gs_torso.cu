// The GS decoder torso's two non-GEMM operations (gs_decoder_graph.cpp:13-155):
//
//   s3dsp_gather_rows      y[i] = x[rows[i]] (ggml_get_rows with the window
//                          tables' bucket order, :64) with a dtype conversion
//   s3dsp_window_attention softmax(q k^T * scale) v within each Swin window,
//                          per head, the bucket loop of :88-118; the result
//                          rows go back to token order (get_rows by bwd_idx,
//                          :121) by writing row i to out[scatter[i]]
//
// Windows are runs of consecutive rows in bucket order (start, len): every
// window of a bucket holds `len` tokens (GsTables::build, sparse_ops.cpp:
// 182-270). Attention runs in f32 whatever the precision of the Linears
// around it: one CTA per (window, head), 128 threads, each thread owning one
// query row of the window per pass; keys and values are staged through
// shared memory in chunks of 64 rows. Per query the softmax is evaluated in
// the reference's order: the row maximum of the scaled scores first, then
// exp(s - max), their sum, and the value rows weighted by exp(s - max) / sum.
#include "s3dsp_internal.h"

using namespace s3dsp;

namespace {

constexpr int kKeyChunk = 64;

__device__ __forceinline__ float ld_any(const void* p, uint32_t dt, int64_t i) {
    if (dt == S3DSP_F32) return reinterpret_cast<const float*>(p)[i];
    if (dt == S3DSP_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    return __half2float(reinterpret_cast<const __half*>(p)[i]);
}
__device__ __forceinline__ void st_any(void* p, uint32_t dt, int64_t i, float v) {
    if (dt == S3DSP_F32)
        reinterpret_cast<float*>(p)[i] = v;
    else if (dt == S3DSP_BF16)
        reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16(v);
    else
        reinterpret_cast<__half*>(p)[i] = __float2half(v);
}

// y[i, :] = x[rows[i], :]; a row index outside [0, n_in) gives zeros and sets kErrRowRange
__global__ void gather_rows_kernel(const void* __restrict__ x, uint32_t xd, int64_t n_in, int64_t c,
                                   const int32_t* __restrict__ rows, int64_t n_out, void* __restrict__ y, uint32_t yd,
                                   uint32_t* __restrict__ status) {
    pdl_wait();
    pdl_trigger();
    const int64_t total = n_out * c;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / c, k = i - r * c;
        const int32_t s = __ldg(rows + r);
        float v = 0.f;
        if (s >= 0 && s < n_in)
            v = ld_any(x, xd, (int64_t)s * c + k);
        else if (k == 0)
            atomicOr(status, kErrRowRange);
        st_any(y, yd, i, v);
    }
}

// One window of one head, one query row per thread and pass (the path for
// windows longer than kMaxWindow): keys and values staged through shared
// memory in chunks of 64 rows (sk, sv: [kKeyChunk][D] each); per query the row
// maximum of the scaled scores first, then exp(s - max), their sum and the
// value rows weighted by exp(s - max), divided by the sum at the end.
template <int D, int kThreads>
__device__ __forceinline__ void attend_per_query(const float* __restrict__ qkv, int64_t n, int c, int64_t start,
                                                 int len, int h, float scale, const int32_t* __restrict__ scatter,
                                                 float* __restrict__ out, uint32_t* __restrict__ status,
                                                 float (*sk)[D], float (*sv)[D]) {
    const int64_t ld = 3 * (int64_t)c;
    const int passes = (len + kThreads - 1) / kThreads;
    for (int pass = 0; pass < passes; ++pass) {
        const int qi = pass * kThreads + threadIdx.x;
        const bool have_q = qi < len;
        float q[D];
        if (have_q) {
            const float4* qrow = reinterpret_cast<const float4*>(qkv + (start + qi) * ld + (int64_t)h * D);
#pragma unroll
            for (int j = 0; j < D / 4; ++j) {
                const float4 t = __ldg(qrow + j);
                q[4 * j] = t.x, q[4 * j + 1] = t.y, q[4 * j + 2] = t.z, q[4 * j + 3] = t.w;
            }
        }
        // sweep 0: the row maximum of the scaled scores; sweep 1: exp sums and the weighted values
        float mx = -INFINITY, sum = 0.f;
        float acc[D];
#pragma unroll
        for (int j = 0; j < D; ++j) acc[j] = 0.f;
        for (int sweep = 0; sweep < 2; ++sweep) {
            for (int k0 = 0; k0 < len; k0 += kKeyChunk) {
                const int kn = min(kKeyChunk, len - k0);
                __syncthreads();
                for (int e = threadIdx.x; e < kn * (D / 4); e += kThreads) {
                    const int r = e / (D / 4), j = e - r * (D / 4);
                    const float* row = qkv + (start + k0 + r) * ld + (int64_t)h * D + 4 * j;
                    *reinterpret_cast<float4*>(&sk[r][4 * j]) = __ldg(reinterpret_cast<const float4*>(row + c));
                    if (sweep == 1)
                        *reinterpret_cast<float4*>(&sv[r][4 * j]) = __ldg(reinterpret_cast<const float4*>(row + 2 * c));
                }
                __syncthreads();
                if (!have_q) continue;
                for (int r = 0; r < kn; ++r) {
                    float dot = 0.f;
#pragma unroll
                    for (int j = 0; j < D; ++j) dot = fmaf(q[j], sk[r][j], dot);
                    const float s = dot * scale;
                    if (sweep == 0) {
                        mx = fmaxf(mx, s);
                    } else {
                        const float p = expf(s - mx);
                        sum += p;
#pragma unroll
                        for (int j = 0; j < D; ++j) acc[j] = fmaf(p, sv[r][j], acc[j]);
                    }
                }
            }
        }
        if (have_q) {
            const int64_t orow = scatter ? (int64_t)scatter[start + qi] : start + qi;
            if (orow < 0 || orow >= n) {
                atomicOr(status, kErrRowRange);
            } else {
                const float inv = 1.0f / sum;
                float4* dst = reinterpret_cast<float4*>(out + orow * (int64_t)c + (int64_t)h * D);
#pragma unroll
                for (int j = 0; j < D / 4; ++j)
                    dst[j] = make_float4(acc[4 * j] * inv, acc[4 * j + 1] * inv, acc[4 * j + 2] * inv,
                                         acc[4 * j + 3] * inv);
            }
        }
    }
}

// Tiled form, one CTA per (window, head), windows of at most kMaxWindow rows,
// 64 queries at a time:
//  1. S = (Q K^T) * scale in 4 x 4 register blocks per thread (the dot over the
//     head's channels in channel order), kept key-major in shared memory;
//  2. the softmax in the reference's order: the row maximum, then
//     exp(s - max) in place, then one thread per query sums them in key order;
//  3. O = P V in 4 x (D / 16) register blocks, accumulated in key order, times
//     1 / sum.
// Every score, sum and accumulation is evaluated in the same order as in
// attend_per_query, so both give the same bits; longer windows take that path
// (the window tables of a 64^3 shell hold at most ~235 tokens per window).
// About 97 KB of shared memory and at most 128 registers: two CTAs per SM.
constexpr int kTileThreads = 256;
constexpr int kQB = 64;          // queries per block, and keys per chunk
constexpr int kMaxWindow = 256;  // score rows kept in shared memory: two CTAs per SM

template <int D>
constexpr size_t tiled_smem_bytes() {
    return sizeof(float) * ((size_t)kMaxWindow * kQB + 2 * (size_t)D * kQB + 5 * (size_t)kQB);
}

template <int D>
__global__ void __launch_bounds__(kTileThreads, 2)
    window_attention_tiled_kernel(const float* __restrict__ qkv, int64_t n, int c, const int2* __restrict__ windows,
                                  float scale, const int32_t* __restrict__ scatter, float* __restrict__ out,
                                  uint32_t* __restrict__ status) {
    pdl_wait();
    pdl_trigger();
    constexpr int DPT = D / 16;  // output channels per thread in phase 3
    extern __shared__ __align__(16) float sm[];
    float* St = sm;                          // [kMaxWindow][kQB] scores, then exp(s - max)
    float* Qt = St + kMaxWindow * kQB;       // [D][kQB] the query block, transposed
    float* Kt = Qt + D * kQB;                // [D][kQB] a key chunk, transposed (phase 1)
    float* Vs = Kt;                          // [kQB][D] a value chunk (phase 3, same space)
    float* pmax = Kt + D * kQB;              // [4][kQB] partial row maxima
    float* inv = pmax + 4 * kQB;             // [kQB] 1 / sum
    const int2 w = windows[blockIdx.x];
    const int h = blockIdx.y;
    const int64_t start = w.x;
    const int len = w.y;
    if (start < 0 || len <= 0 || start + len > n) {
        if (threadIdx.x == 0) atomicOr(status, kErrRowRange);
        return;
    }
    if (len > kMaxWindow) {
        attend_per_query<D, kTileThreads>(qkv, n, c, start, len, h, scale, scatter, out, status,
                                          reinterpret_cast<float(*)[D]>(Qt), reinterpret_cast<float(*)[D]>(Kt));
        return;
    }
    const int64_t ld = 3 * (int64_t)c;
    const float* base = qkv + start * ld + (int64_t)h * D;  // q of the window's first row
    const int tid = threadIdx.x;
    const int ti = tid & 15;   // queries 4 ti .. 4 ti + 3
    const int tr = tid >> 4;   // phase 1: keys 4 tr ..; phase 3: channels DPT tr ..
    for (int q0 = 0; q0 < len; q0 += kQB) {
        const int qn = min(kQB, len - q0);
        __syncthreads();  // the previous block is done with St, Qt, Vs and inv
        for (int e = tid; e < kQB * (D / 4); e += kTileThreads) {
            const int i = e % kQB, j4 = e / kQB;  // a warp: 32 consecutive rows (no bank conflicts)
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (i < qn) v = __ldg(reinterpret_cast<const float4*>(base + (q0 + i) * ld + 4 * j4));
            Qt[(4 * j4 + 0) * kQB + i] = v.x;
            Qt[(4 * j4 + 1) * kQB + i] = v.y;
            Qt[(4 * j4 + 2) * kQB + i] = v.z;
            Qt[(4 * j4 + 3) * kQB + i] = v.w;
        }
        // ---- phase 1: scaled scores ----
        for (int k0 = 0; k0 < len; k0 += kQB) {
            const int kn = min(kQB, len - k0);
            __syncthreads();  // Kt is free (and Qt complete)
            for (int e = tid; e < kQB * (D / 4); e += kTileThreads) {
                const int r = e % kQB, j4 = e / kQB;
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (r < kn) v = __ldg(reinterpret_cast<const float4*>(base + (k0 + r) * ld + c + 4 * j4));
                Kt[(4 * j4 + 0) * kQB + r] = v.x;
                Kt[(4 * j4 + 1) * kQB + r] = v.y;
                Kt[(4 * j4 + 2) * kQB + r] = v.z;
                Kt[(4 * j4 + 3) * kQB + r] = v.w;
            }
            __syncthreads();
            float acc[4][4];
#pragma unroll
            for (int x = 0; x < 4; ++x)
#pragma unroll
                for (int y = 0; y < 4; ++y) acc[x][y] = 0.f;
#pragma unroll 8
            for (int j = 0; j < D; ++j) {
                const float4 a = *reinterpret_cast<const float4*>(Qt + j * kQB + 4 * ti);
                const float4 b = *reinterpret_cast<const float4*>(Kt + j * kQB + 4 * tr);
                const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
                for (int x = 0; x < 4; ++x)
#pragma unroll
                    for (int y = 0; y < 4; y += 2) fma2(acc[x][y], acc[x][y + 1], av[x], bv[y], bv[y + 1]);
            }
#pragma unroll
            for (int y = 0; y < 4; ++y) {
                const int r = 4 * tr + y;
                if (r < kn)
                    *reinterpret_cast<float4*>(St + (k0 + r) * kQB + 4 * ti) =
                        make_float4(acc[0][y] * scale, acc[1][y] * scale, acc[2][y] * scale, acc[3][y] * scale);
            }
        }
        __syncthreads();
        // ---- phase 2: the softmax (maximum, exp(s - max), sum in key order) ----
        {
            const int i = tid & (kQB - 1), part = tid / kQB;  // four threads per query
            float m = -INFINITY;
            for (int r = part; r < len; r += 4) m = fmaxf(m, St[r * kQB + i]);
            pmax[part * kQB + i] = m;
            __syncthreads();
            const float mx = fmaxf(fmaxf(pmax[i], pmax[kQB + i]), fmaxf(pmax[2 * kQB + i], pmax[3 * kQB + i]));
            for (int r = part; r < len; r += 4) St[r * kQB + i] = expf(St[r * kQB + i] - mx);
            __syncthreads();
            if (tid < kQB) {
                float sum = 0.f;
                for (int r = 0; r < len; ++r) sum += St[r * kQB + tid];
                inv[tid] = 1.0f / sum;
            }
        }
        // ---- phase 3: O = P V ----
        float o[4][DPT];
#pragma unroll
        for (int x = 0; x < 4; ++x)
#pragma unroll
            for (int y = 0; y < DPT; ++y) o[x][y] = 0.f;
        for (int k0 = 0; k0 < len; k0 += kQB) {
            const int kn = min(kQB, len - k0);
            __syncthreads();  // Vs is free (and the sums are done)
            for (int e = tid; e < kn * (D / 4); e += kTileThreads) {
                const int r = e / (D / 4), j4 = e % (D / 4);
                *reinterpret_cast<float4*>(Vs + r * D + 4 * j4) =
                    __ldg(reinterpret_cast<const float4*>(base + (k0 + r) * ld + 2 * c + 4 * j4));
            }
            __syncthreads();
            for (int r = 0; r < kn; ++r) {
                const float4 p4 = *reinterpret_cast<const float4*>(St + (k0 + r) * kQB + 4 * ti);
                const float pv[4] = {p4.x, p4.y, p4.z, p4.w};
                float v[DPT];
#pragma unroll
                for (int y = 0; y < DPT; ++y) v[y] = Vs[r * D + DPT * tr + y];
#pragma unroll
                for (int x = 0; x < 4; ++x)
#pragma unroll
                    for (int y = 0; y < DPT; y += 2) fma2(o[x][y], o[x][y + 1], pv[x], v[y], v[y + 1]);
            }
        }
#pragma unroll
        for (int x = 0; x < 4; ++x) {
            const int i = 4 * ti + x;
            if (i >= qn) continue;
            const int64_t orow = scatter ? (int64_t)scatter[start + q0 + i] : start + q0 + i;
            if (orow < 0 || orow >= n) {
                atomicOr(status, kErrRowRange);
                continue;
            }
            float* dst = out + orow * (int64_t)c + (int64_t)h * D + DPT * tr;
#pragma unroll
            for (int y = 0; y < DPT; ++y) dst[y] = o[x][y] * inv[i];
        }
    }
}

int grid_for_rows(int64_t work, int sm_count) {
    int64_t g = (work + 255) / 256;
    if (g > (int64_t)sm_count * 16) g = (int64_t)sm_count * 16;
    return (int)(g < 1 ? 1 : g);
}

}  // namespace

extern "C" S3DSP_API s3d_status s3dsp_gather_rows(s3dsp_context* ctx, const void* x, uint32_t x_dtype, int64_t n_in,
                                                  int64_t c, const int32_t* d_rows, int64_t n_out, void* y,
                                                  uint32_t y_dtype, char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !x || !d_rows || !y) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    if (!dtype_ok(x_dtype) || !dtype_ok(y_dtype) || n_in < 0 || n_out < 0 || c <= 0)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "bad shape/dtype");
    if (n_out == 0) return S3D_OK;
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    S3DSP_CUDA(launch_pdl(gather_rows_kernel, dim3(grid_for_rows(n_out * c, ctx->sm_count)), dim3(256), 0, ctx->stream,
                          x, x_dtype, n_in, c, d_rows, n_out, y, y_dtype, ctx->d_status),
               "gather_rows_kernel");
    return S3D_OK;
}

extern "C" S3DSP_API s3d_status s3dsp_window_attention(s3dsp_context* ctx, const float* qkv, int64_t n, int64_t c,
                                                       int32_t heads, const int32_t* d_windows, int64_t n_windows,
                                                       const int32_t* d_scatter, float* out, char* error,
                                                       uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !qkv || !out || (n_windows > 0 && !d_windows))
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    if (n < 0 || c <= 0 || heads <= 0 || c % heads || n_windows < 0 || n_windows > 0x7fffffff)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "bad shape");
    const int64_t d = c / heads;
    if (d != 32 && d != 64)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "head dimension %lld (32 or 64 supported)",
                    (long long)d);
    if (((uintptr_t)qkv & 15) || ((uintptr_t)out & 15))
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "qkv and out need 16-byte alignment");
    if (n_windows == 0 || n == 0) return S3D_OK;
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    const dim3 grid((unsigned)n_windows, (unsigned)heads);
    const float scale = 1.0f / sqrtf((float)d);
    const int2* win = reinterpret_cast<const int2*>(d_windows);
    cudaError_t e;
    static std::atomic<uint64_t> optin32{0}, optin64{0};
    if (d == 32) {
        e = smem_optin((const void*)window_attention_tiled_kernel<32>, ctx->device, optin32);
        if (e == cudaSuccess)
            e = launch_pdl(window_attention_tiled_kernel<32>, grid, dim3(kTileThreads), tiled_smem_bytes<32>(),
                           ctx->stream, qkv, n, (int)c, win, scale, d_scatter, out, ctx->d_status);
    } else {
        e = smem_optin((const void*)window_attention_tiled_kernel<64>, ctx->device, optin64);
        if (e == cudaSuccess)
            e = launch_pdl(window_attention_tiled_kernel<64>, grid, dim3(kTileThreads), tiled_smem_bytes<64>(),
                           ctx->stream, qkv, n, (int)c, win, scale, d_scatter, out, ctx->d_status);
    }
    if (e != cudaSuccess) return cuda_fail(error, error_capacity, e, "window_attention_kernel");
    S3DSP_LAUNCH_CHECK("window_attention_kernel");
    return S3D_OK;
}
