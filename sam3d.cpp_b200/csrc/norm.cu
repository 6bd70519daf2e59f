// Normalisation kernels (GroupNorm statistics / finalize / apply, LayerNorm
// with modulate and SiLU), dtype conversion and weight packing.
//
// GroupNorm follows sparse_group_norm (src/objects_runtime/mesh_decoder_graph.cpp
// :16-30): one object, `groups` equal channel ranges, statistics over every
// token, eps 1e-5, then gamma/beta. Statistics are accumulated as per-128-row
// tile partial sums in double ([tiles][groups][2]); the finalize kernel reduces
// them in a fixed order (deterministic) and emits per-channel (sub, mul, add)
// with (x - sub) * mul + add == ((x - mean) * rstd) * gamma + beta.
// LayerNorm follows ggml_norm + mul/add (graph_builder.cpp:56-62) and modulate
// (slat_flow_graph.cpp:55-59): y = silu(((x-mean)*rstd*g + b) * (1+s) + sh).
#include "s3dsp_internal.h"

using namespace s3dsp;

namespace {

__device__ __forceinline__ float ld_f(const void* p, uint32_t dt, int64_t i) {
    if (dt == S3DSP_F32) return reinterpret_cast<const float*>(p)[i];
    if (dt == S3DSP_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    return __half2float(reinterpret_cast<const __half*>(p)[i]);
}
__device__ __forceinline__ void st_f(void* p, uint32_t dt, int64_t i, float v) {
    if (dt == S3DSP_F32)
        reinterpret_cast<float*>(p)[i] = v;
    else if (dt == S3DSP_BF16)
        reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16(v);
    else
        reinterpret_cast<__half*>(p)[i] = __float2half(v);
}
__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + __expf(-v)); }
// for a bf16 result: the approximate divide's error is far below bf16 rounding
// (1 + exp(-v) is >= 1, and +inf for v < -88, where the quotient is 0)
__device__ __forceinline__ float silu_fast(float v) { return __fdividef(v, 1.0f + __expf(-v)); }

// stats of x [n, c]: one block per 128-row tile; block-local double sums per
// group written (not accumulated) to partials[tile][g][2]
__global__ void gn_stats_kernel(const void* __restrict__ x, uint32_t dt, int64_t n, int c, int groups,
                                double* __restrict__ partials) {
    pdl_wait();
    pdl_trigger();
    __shared__ double acc[64][2];
    for (int i = threadIdx.x; i < 128; i += blockDim.x) (&acc[0][0])[i] = 0.0;
    __syncthreads();
    const int gs = c / groups;
    const int64_t r0 = (int64_t)blockIdx.x * 128;
    const int64_t rows = min((int64_t)128, n - r0);
    // thread -> channel column stripe; accumulate per channel then per group
    for (int ch = threadIdx.x; ch < c; ch += blockDim.x) {
        double s1 = 0.0, s2 = 0.0;
        for (int64_t r = 0; r < rows; ++r) {
            const double v = ld_f(x, dt, (r0 + r) * c + ch);
            s1 += v;
            s2 += v * v;
        }
        atomicAdd(&acc[ch / gs][0], s1);
        atomicAdd(&acc[ch / gs][1], s2);
    }
    __syncthreads();
    for (int g = threadIdx.x; g < groups; g += blockDim.x) {
        partials[((int64_t)blockIdx.x * groups + g) * 2 + 0] = acc[g][0];
        partials[((int64_t)blockIdx.x * groups + g) * 2 + 1] = acc[g][1];
    }
}

// one block per group: fixed-order tree reduction over tiles
__global__ void gn_finalize_kernel(const double* __restrict__ partials, int64_t tiles, int64_t n_rows, int c,
                                   int groups, float eps, const float* __restrict__ gamma,
                                   const float* __restrict__ beta, float* __restrict__ sub, float* __restrict__ mul,
                                   float* __restrict__ add) {
    pdl_wait();
    pdl_trigger();
    __shared__ double s1s[256], s2s[256];
    const int g = blockIdx.x;
    double s1 = 0.0, s2 = 0.0;
    for (int64_t t = threadIdx.x; t < tiles; t += blockDim.x) {
        s1 += partials[(t * groups + g) * 2 + 0];
        s2 += partials[(t * groups + g) * 2 + 1];
    }
    s1s[threadIdx.x] = s1;
    s2s[threadIdx.x] = s2;
    __syncthreads();
    for (int d = blockDim.x / 2; d > 0; d >>= 1) {
        if ((int)threadIdx.x < d) {
            s1s[threadIdx.x] += s1s[threadIdx.x + d];
            s2s[threadIdx.x] += s2s[threadIdx.x + d];
        }
        __syncthreads();
    }
    const int gs = c / groups;
    if ((int)threadIdx.x < gs) {
        const double cnt = (double)n_rows * (double)gs;
        const double mean = s1s[0] / cnt;
        double var = s2s[0] / cnt - mean * mean;
        if (var < 0.0) var = 0.0;
        const float rstd = 1.0f / sqrtf((float)var + eps);
        const int ch = g * gs + threadIdx.x;
        const float gm = gamma ? gamma[ch] : 1.0f;
        sub[ch] = (float)mean;
        mul[ch] = rstd * gm;
        add[ch] = beta ? beta[ch] : 0.0f;
    }
}

__global__ void channel_affine_kernel(const void* __restrict__ x, uint32_t xd, int64_t n, int c,
                                      const float* __restrict__ sub, const float* __restrict__ mul,
                                      const float* __restrict__ add, int silu, void* __restrict__ y, uint32_t yd) {
    pdl_wait();
    pdl_trigger();
    const int64_t total = n * c;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int ch = (int)(i % c);
        float v = (ld_f(x, xd, i) - sub[ch]) * mul[ch] + add[ch];
        if (silu) v = silu_f(v);
        st_f(y, yd, i, v);
    }
}

// vectorised variant: f32 or bf16 in, bf16 out, c % 8 == 0
// x -> affine (+SiLU) -> bf16, 8 channels per item, 4 items per thread per
// iteration with all loads issued before any use (bytes in flight per SM is
// what bounds a streaming kernel). (x - sub) * mul + add is evaluated as
// written, with the per-channel vectors read as float4.
template <typename InT>
__device__ __forceinline__ void load8(const void* x, int64_t i, float (&v)[8]);
template <>
__device__ __forceinline__ void load8<float>(const void* x, int64_t i, float (&v)[8]) {
    const float4 a = __ldcs(reinterpret_cast<const float4*>(x) + 2 * i);
    const float4 b = __ldcs(reinterpret_cast<const float4*>(x) + 2 * i + 1);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const void* x, int64_t i, float (&v)[8]) {
    const uint4 u = __ldcs(reinterpret_cast<const uint4*>(x) + i);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[q]));
        v[2 * q] = f.x;
        v[2 * q + 1] = f.y;
    }
}

template <typename InT>
__global__ void channel_affine_bf16_out_kernel(const void* __restrict__ x, int64_t total8, uint32_t c8,
                                               const float4* __restrict__ sub, const float4* __restrict__ mul,
                                               const float4* __restrict__ add, int silu, uint4* __restrict__ y) {
    pdl_wait();
    pdl_trigger();
    constexpr int U = 4;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const bool narrow = total8 <= 0xffffffffll;
    for (int64_t i0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i0 < total8; i0 += stride * U) {
        float a[U][8];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t i = i0 + u * stride;
            if (i < total8) load8<InT>(x, i, a[u]);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t i = i0 + u * stride;
            if (i >= total8) break;
            // 8-channel group within the row (32-bit remainder when the index fits)
            const uint32_t q8 = narrow ? (uint32_t)i % c8 : (uint32_t)((uint64_t)i % c8);
            const float4 s0 = __ldg(sub + 2 * q8), s1 = __ldg(sub + 2 * q8 + 1);
            const float4 m0 = __ldg(mul + 2 * q8), m1 = __ldg(mul + 2 * q8 + 1);
            const float4 d0 = __ldg(add + 2 * q8), d1 = __ldg(add + 2 * q8 + 1);
            float v[8] = {(a[u][0] - s0.x) * m0.x + d0.x, (a[u][1] - s0.y) * m0.y + d0.y,
                          (a[u][2] - s0.z) * m0.z + d0.z, (a[u][3] - s0.w) * m0.w + d0.w,
                          (a[u][4] - s1.x) * m1.x + d1.x, (a[u][5] - s1.y) * m1.y + d1.y,
                          (a[u][6] - s1.z) * m1.z + d1.z, (a[u][7] - s1.w) * m1.w + d1.w};
            if (silu) {
#pragma unroll
                for (int q = 0; q < 8; ++q) v[q] = silu_fast(v[q]);
            }
            uint32_t w[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * q], v[2 * q + 1]);
                w[q] = *reinterpret_cast<const uint32_t*>(&h);
            }
            y[i] = make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
}

// one warp per row; two passes over the row (mean, then centred variance),
// both in double like ggml_norm's ggml_float sums
// x: one source [n, c], or the channel concat of xa [n, ca] and xb [n, c - ca]
// (xb non-null); y [n, c]
__global__ void layer_norm_kernel(const void* __restrict__ x, const void* __restrict__ xb, int ca, uint32_t xd,
                                  int64_t n, int c, float eps, const float* __restrict__ gamma,
                                  const float* __restrict__ beta, const float* __restrict__ ms,
                                  const float* __restrict__ msh, int silu, void* __restrict__ y, uint32_t yd) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int64_t row = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= n) return;
    const int cb = c - ca;
    auto ld = [&](int k) {
        return k < ca ? ld_f(x, xd, row * ca + k) : ld_f(xb, xd, row * cb + (k - ca));
    };
    double s = 0.0;
    for (int k = lane; k < c; k += 32) s += ld(k);
    for (int d = 16; d > 0; d >>= 1) s += __shfl_xor_sync(0xffffffffu, s, d);
    const float mean = (float)(s / c);
    double s2 = 0.0;
    for (int k = lane; k < c; k += 32) {
        const float v = ld(k) - mean;
        s2 += (double)v * v;
    }
    for (int d = 16; d > 0; d >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, d);
    const float rstd = 1.0f / sqrtf((float)(s2 / c) + eps);
    const int64_t base = row * c;
    for (int k = lane; k < c; k += 32) {
        float v = (ld(k) - mean) * rstd;
        if (gamma) v *= gamma[k];
        if (beta) v += beta[k];
        if (ms) v = v * ms[k] + v;
        if (msh) v += msh[k];
        if (silu) v = silu_f(v);
        st_f(y, yd, base + k, v);
    }
}

__global__ void convert_kernel(const void* __restrict__ x, uint32_t xd, void* __restrict__ y, uint32_t yd,
                               int64_t count) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x)
        st_f(y, yd, i, ld_f(x, xd, i));
}

// f32 -> bf16, 4 elements per item, 4 items per thread per iteration (loads first)
__global__ void convert_f32_bf16_kernel(const float4* __restrict__ x, uint2* __restrict__ y, int64_t count4) {
    pdl_wait();
    pdl_trigger();
    constexpr int U = 4;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i0 < count4; i0 += stride * U) {
        float4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (i0 + u * stride < count4) v[u] = __ldg(x + i0 + u * stride);
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t i = i0 + u * stride;
            if (i >= count4) break;
            const __nv_bfloat162 a = __floats2bfloat162_rn(v[u].x, v[u].y), b = __floats2bfloat162_rn(v[u].z, v[u].w);
            y[i] = make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
        }
    }
}

// Weight packing. Source element (o, co, ci) of each layout, as stored in GGUF:
//   SLAT_ROW      (Cout, 27, Cin)      src[(co*kvol + o)*cin + ci]
//   MESH_PACKED   (kvol, Cout, Cin)    src[(o*cout + co)*cin + ci]
//   LINEAR        (Cout, Cin), kvol 1  src[co*cin + ci]
//   SPCONV_1X1    buffer read as (Cin, Cout) then transposed: src[ci*cout + co]
//   TRANSPOSED_2X2X2 (8, Cout, Cin) == MESH_PACKED with kvol 8
// Destinations: F32_STRICT -> [kvol][cin_pad16][cout_pad64] f32 (zero padded)
//               BF16       -> [kvol][cout_pad16][cin_pad64] bf16 (K-major)
// x = hi + lo: hi = x rounded to TF32 (10 explicit mantissa bits, ties away
// from zero), lo = x - hi exactly in f32 (zero for non-finite x)
__device__ __forceinline__ void tf32_split(float x, float& hi, float& lo) {
    uint32_t h;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(x));
    hi = __uint_as_float(h);
    lo = isfinite(x) ? __fsub_rn(x, hi) : 0.0f;
}

__global__ void pack_kernel(const void* __restrict__ src, uint32_t sd, uint32_t layout, int kvol, int cin,
                            int cout, uint32_t prec, int cin_pad, int cout_pad, void* __restrict__ dst) {
    pdl_wait();
    pdl_trigger();
    const int64_t total = (int64_t)kvol * cin_pad * cout_pad;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int o, ci, co;
        if (prec == S3DSP_PREC_F32_STRICT) {
            co = (int)(i % cout_pad);
            ci = (int)((i / cout_pad) % cin_pad);
            o = (int)(i / ((int64_t)cout_pad * cin_pad));
        } else {
            ci = (int)(i % cin_pad);
            co = (int)((i / cin_pad) % cout_pad);
            o = (int)(i / ((int64_t)cout_pad * cin_pad));
        }
        float v = 0.0f;
        if (ci < cin && co < cout) {
            int64_t s;
            switch (layout) {
                case S3DSP_LAYOUT_SLAT_ROW: s = ((int64_t)co * kvol + o) * cin + ci; break;
                case S3DSP_LAYOUT_SPCONV_1X1: s = (int64_t)ci * cout + co; break;
                case S3DSP_LAYOUT_LINEAR: s = (int64_t)co * cin + ci; break;
                default: s = ((int64_t)o * cout + co) * cin + ci; break;  // MESH_PACKED / TRANSPOSED
            }
            v = ld_f(src, sd, s);
        }
        if (prec == S3DSP_PREC_F32_STRICT) {
            reinterpret_cast<float*>(dst)[i] = v;
        } else if (prec == S3DSP_PREC_F32_3XTF32) {
            // high block [kvol][cout_pad][cin_pad] then the low block of remainders
            float hi, lo;
            tf32_split(v, hi, lo);
            reinterpret_cast<float*>(dst)[i] = hi;
            reinterpret_cast<float*>(dst)[i + total] = lo;
        } else {
            reinterpret_cast<__nv_bfloat16*>(dst)[i] = __float2bfloat16(v);
        }
    }
}

__global__ void split_tf32_kernel(const float* __restrict__ x, int64_t n, float* __restrict__ hi,
                                  float* __restrict__ lo) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        float h, l;
        tf32_split(__ldg(x + i), h, l);
        hi[i] = h;
        lo[i] = l;
    }
}

inline int grid_for(int64_t n, int threads, int sm_count) {
    int64_t g = (n + threads - 1) / threads;
    const int64_t cap = (int64_t)sm_count * 16;
    if (g > cap) g = cap;
    return (int)(g < 1 ? 1 : g);
}

}  // namespace

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
extern "C" S3DSP_API int64_t s3dsp_gn_partials_count(int64_t n_rows, int64_t channels, int32_t groups) {
    (void)channels;
    return ((n_rows + 127) / 128) * (int64_t)groups * 2;
}

extern "C" S3DSP_API s3d_status s3dsp_gn_stats(s3dsp_context* ctx, const void* x, uint32_t dtype, int64_t n,
                                               int64_t c, int32_t groups, double* partials, char* error,
                                               uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !x || !partials) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    if (!dtype_ok(dtype) || n <= 0 || c <= 0 || groups <= 0 || groups > 64 || c % groups)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "bad GroupNorm shape n=%lld c=%lld groups=%d",
                    (long long)n, (long long)c, groups);
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    const int64_t tiles = (n + 127) / 128;
    launch_pdl(gn_stats_kernel, dim3((unsigned)tiles), dim3(256), 0, ctx->stream, x, dtype, n, (int)c, groups,
               partials);
    S3DSP_LAUNCH_CHECK("gn_stats_kernel");
    return S3D_OK;
}

extern "C" S3DSP_API s3d_status s3dsp_gn_finalize(s3dsp_context* ctx, const double* partials, int64_t n_rows,
                                                  int64_t c, int32_t groups, float eps, const float* gamma,
                                                  const float* beta, float* sub, float* mul, float* add,
                                                  char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !partials || !sub || !mul || !add)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    if (n_rows <= 0 || c <= 0 || groups <= 0 || groups > 64 || c % groups || c / groups > 256)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "bad GroupNorm shape");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    S3DSP_CUDA(launch_pdl(gn_finalize_kernel, dim3(groups), dim3(256), 0, ctx->stream, partials,
                          (int64_t)((n_rows + 127) / 128), n_rows, (int)c, (int)groups, eps, gamma, beta, sub, mul, add),
               "gn_finalize_kernel");
    S3DSP_LAUNCH_CHECK("gn_finalize_kernel");
    return S3D_OK;
}

extern "C" S3DSP_API s3d_status s3dsp_channel_affine(s3dsp_context* ctx, const void* x, uint32_t xd, int64_t n,
                                                     int64_t c, const float* sub, const float* mul,
                                                     const float* add, int32_t silu, void* y, uint32_t yd,
                                                     char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !x || !y || !sub || !mul || !add)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    if (!dtype_ok(xd) || !dtype_ok(yd) || n < 0 || c <= 0)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "bad shape/dtype");
    if (n == 0) return S3D_OK;
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    const bool vec_ok = !((uintptr_t)x & 15) && !((uintptr_t)y & 15) && !((uintptr_t)sub & 15) &&
                        !((uintptr_t)mul & 15) && !((uintptr_t)add & 15);
    if ((xd == S3DSP_F32 || xd == S3DSP_BF16) && yd == S3DSP_BF16 && c % 8 == 0 && vec_ok) {
        const int64_t total8 = n * c / 8;
        const dim3 grid(grid_for((total8 + 3) / 4, 256, ctx->sm_count));
        auto kern = xd == S3DSP_F32 ? channel_affine_bf16_out_kernel<float> : channel_affine_bf16_out_kernel<__nv_bfloat16>;
        S3DSP_CUDA(launch_pdl(kern, grid, dim3(256), 0, ctx->stream, x, total8, (uint32_t)(c / 8),
                              reinterpret_cast<const float4*>(sub), reinterpret_cast<const float4*>(mul),
                              reinterpret_cast<const float4*>(add), (int)silu, reinterpret_cast<uint4*>(y)),
                   "channel_affine_bf16_out_kernel");
    } else {
        launch_pdl(channel_affine_kernel, dim3(grid_for(n * c, 256, ctx->sm_count)), dim3(256), 0, ctx->stream, x, xd,
                   n, (int)c, sub, mul, add, silu, y, yd);
    }
    S3DSP_LAUNCH_CHECK("channel_affine_kernel");
    return S3D_OK;
}

extern "C" S3DSP_API s3d_status s3dsp_layer_norm(s3dsp_context* ctx, const void* x, uint32_t xd, int64_t n, int64_t c,
                                                 float eps, const float* gamma, const float* beta,
                                                 const float* ms, const float* msh, int32_t silu, void* y,
                                                 uint32_t yd, char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !x || !y) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    if (!dtype_ok(xd) || !dtype_ok(yd) || n < 0 || c <= 0)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "bad shape/dtype");
    if (n == 0) return S3D_OK;
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    const int64_t blocks = (n + 7) / 8;
    launch_pdl(layer_norm_kernel, dim3((unsigned)blocks), dim3(256), 0, ctx->stream, x, (const void*)nullptr, (int)c,
               xd, n, (int)c, eps, gamma, beta, ms, msh, silu, y, yd);
    S3DSP_LAUNCH_CHECK("layer_norm_kernel");
    return S3D_OK;
}

extern "C" S3DSP_API s3d_status s3dsp_layer_norm_concat(s3dsp_context* ctx, const void* xa, int64_t ca,
                                                        const void* xb, int64_t cb, uint32_t xd, int64_t n, float eps,
                                                        const float* gamma, const float* beta, const float* ms,
                                                        const float* msh, int32_t silu, void* y, uint32_t yd,
                                                        char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !xa || !xb || !y) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    if (!dtype_ok(xd) || !dtype_ok(yd) || n < 0 || ca <= 0 || cb <= 0 || ca + cb > (1 << 20))
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "bad shape/dtype");
    if (n == 0) return S3D_OK;
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    const int64_t blocks = (n + 7) / 8;
    launch_pdl(layer_norm_kernel, dim3((unsigned)blocks), dim3(256), 0, ctx->stream, xa, xb, (int)ca, xd, n,
               (int)(ca + cb), eps, gamma, beta, ms, msh, silu, y, yd);
    S3DSP_LAUNCH_CHECK("layer_norm_kernel");
    return S3D_OK;
}

extern "C" S3DSP_API s3d_status s3dsp_convert(s3dsp_context* ctx, const void* x, uint32_t xd, void* y, uint32_t yd,
                                              int64_t count, char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !x || !y) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    if (!dtype_ok(xd) || !dtype_ok(yd) || count < 0)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "bad dtype/count");
    if (count == 0) return S3D_OK;
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    if (xd == S3DSP_F32 && yd == S3DSP_BF16 && count % 4 == 0 && !((uintptr_t)x & 15) && !((uintptr_t)y & 7))
        S3DSP_CUDA(launch_pdl(convert_f32_bf16_kernel, dim3(grid_for((count / 4 + 3) / 4, 256, ctx->sm_count)),
                              dim3(256), 0, ctx->stream, reinterpret_cast<const float4*>(x), reinterpret_cast<uint2*>(y),
                              (int64_t)(count / 4)),
                   "convert_f32_bf16_kernel");
    else
        launch_pdl(convert_kernel, dim3(grid_for(count, 256, ctx->sm_count)), dim3(256), 0, ctx->stream, x, xd, y, yd,
                   count);
    S3DSP_LAUNCH_CHECK("convert_kernel");
    return S3D_OK;
}

namespace {
void packed_dims(uint32_t prec, int64_t cin, int64_t cout, int64_t& cin_pad, int64_t& cout_pad) {
    if (prec == S3DSP_PREC_F32_STRICT) {
        cin_pad = (cin + 15) / 16 * 16;
        cout_pad = (cout + 63) / 64 * 64;
    } else if (prec == S3DSP_PREC_F32_3XTF32) {
        cin_pad = (cin + 31) / 32 * 32;
        cout_pad = (cout + 15) / 16 * 16;
    } else {
        cin_pad = (cin + 63) / 64 * 64;
        cout_pad = (cout + 15) / 16 * 16;
    }
}
}  // namespace

extern "C" S3DSP_API int64_t s3dsp_weights_packed_bytes(uint32_t prec, int32_t kvol, int64_t cin, int64_t cout) {
    int64_t cp, op;
    packed_dims(prec, cin, cout, cp, op);
    return (int64_t)kvol * cp * op * (prec == S3DSP_PREC_F32_STRICT ? 4 : prec == S3DSP_PREC_F32_3XTF32 ? 8 : 2);
}

extern "C" S3DSP_API s3d_status s3dsp_weights_pack(s3dsp_context* ctx, const void* src, uint32_t sd, int32_t on_host,
                                                   uint32_t layout, int32_t kvol, int64_t cin, int64_t cout,
                                                   uint32_t prec, void* dst, char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !src || !dst) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    if (!dtype_ok(sd)) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "bad source dtype");
    if (prec != S3DSP_PREC_F32_STRICT && prec != S3DSP_PREC_BF16 && prec != S3DSP_PREC_F32_3XTF32)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "unknown precision %u", prec);
    if (layout > S3DSP_LAYOUT_TRANSPOSED_2X2X2) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "unknown layout");
    if (cin <= 0 || cout <= 0 || (kvol != 1 && kvol != 8 && kvol != 27))
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "bad weight shape");
    if ((layout == S3DSP_LAYOUT_LINEAR || layout == S3DSP_LAYOUT_SPCONV_1X1) && kvol != 1)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "linear layouts need kvol 1");
    if (layout == S3DSP_LAYOUT_SLAT_ROW && kvol != 27)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "SLAT_ROW layout needs kvol 27");
    if (layout == S3DSP_LAYOUT_TRANSPOSED_2X2X2 && kvol != 8)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "TRANSPOSED_2X2X2 layout needs kvol 8");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    int64_t cp, op;
    packed_dims(prec, cin, cout, cp, op);
    const void* dsrc = src;
    void* staged = nullptr;
    if (on_host) {
        const size_t bytes = (size_t)kvol * cin * cout * dtype_size(sd);
        S3DSP_CUDA(s3dsp::malloc_async(&staged, bytes, ctx->stream), "weight staging");
        cudaError_t e = cudaMemcpyAsync(staged, src, bytes, cudaMemcpyHostToDevice, ctx->stream);
        if (e != cudaSuccess) {
            cudaFreeAsync(staged, ctx->stream);
            return cuda_fail(error, error_capacity, e, "weight upload");
        }
        dsrc = staged;
    }
    const int64_t total = (int64_t)kvol * cp * op;
    launch_pdl(pack_kernel, dim3(grid_for(total, 256, ctx->sm_count)), dim3(256), 0, ctx->stream, dsrc, sd, layout,
               kvol, (int)cin, (int)cout, prec, (int)cp, (int)op, dst);
    cudaError_t e = cudaGetLastError();
    if (staged) cudaFreeAsync(staged, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(error, error_capacity, e, "pack_kernel");
    if (on_host) S3DSP_CUDA(cudaStreamSynchronize(ctx->stream), "weight upload sync");
    return S3D_OK;
}

namespace s3dsp {
cudaError_t split_tf32(s3dsp_context* ctx, const float* x, int64_t n, float* hi, float* lo) {
    if (n <= 0) return cudaSuccess;
    launch_pdl(split_tf32_kernel, dim3(grid_for(n, 256, ctx->sm_count)), dim3(256), 0, ctx->stream, x, n, hi, lo);
    return cudaGetLastError();
}
}  // namespace s3dsp
