// F32-strict implicit-gather sparse convolution on the FP32 pipes.
//
// out[r, :] = sum_{o active} sum_ci pro(in[nbr_o(r) >> in_shift, ci]) * W[o, ci, :]
//             + bias (+ residual) (-> SiLU)
// One CTA owns a 128-row x BN-column output tile and walks (offset, 16-channel
// chunk) steps; gathered rows are staged through registers into shared memory
// (transposed, so each thread reads 4 consecutive rows as one float4), double
// buffered. Outputs are accumulated in registers, no atomics. Offsets with no
// neighbour in the tile (per-tile bitmask from the kmap) are skipped.
//
// Replaces the f32 GGML get_rows + mul_mat chains of slat_flow_graph.cpp:
// 112-155 and mesh_decoder_graph.cpp:81-103; the optional prologue applies
// GroupNorm+SiLU of the previous layer to the gathered rows
// (mesh_decoder_graph.cpp:117-121), leaving missing neighbours at zero as the
// reference's mask multiply does (:97-98).
#include "s3dsp_internal.h"

using namespace s3dsp;

namespace {

constexpr int BM = 128;
constexpr int BK = 16;
constexpr int NT = 256;

struct F32ConvParams {
    const float* in;
    const float* in_b;         // second source (channels [cin_a, cin)) or null
    int cin_a;
    int64_t n_in;
    int cin;
    int in_shift;
    const int32_t* nbr;        // [kvol][n_out] or null (identity)
    const uint32_t* tile_mask; // [tiles] or null (all offsets)
    int kvol;
    const float* w;            // packed [kvol][cin_pad][cout_pad]
    int cin_pad, cout_pad;
    const float* bias;
    const void* residual;
    uint32_t res_dtype;
    int res_shift;
    void* out;
    uint32_t out_dtype;
    int64_t n_out;
    int cout;
    uint32_t flags;
    const float* pro_sub;
    const float* pro_mul;
    const float* pro_add;
    double* gn_partials;       // [tiles][groups][2] (zeroed by the launcher)
    int gn_groups;
};

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + __expf(-v)); }

__device__ __forceinline__ float load_as_f32(const void* p, uint32_t dt, int64_t i) {
    if (dt == S3DSP_F32) return reinterpret_cast<const float*>(p)[i];
    if (dt == S3DSP_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    return __half2float(reinterpret_cast<const __half*>(p)[i]);
}

template <int BN>
__global__ void __launch_bounds__(NT) conv_f32_kernel(const F32ConvParams p) {
    pdl_wait();
    pdl_trigger();
    constexpr int TN = BN / 16;
    __shared__ __align__(16) float As[2][BK][BM];
    __shared__ __align__(16) float Bs[2][BK][BN];
    __shared__ double colsum[16][BN][2];  // per row group ty: column sums, summed in a fixed order

    const int tid = threadIdx.x;
    const int64_t m0 = (int64_t)blockIdx.x * BM;
    const int n0 = blockIdx.y * BN;
    const int tile = blockIdx.x;

    uint32_t mask = p.nbr ? (p.tile_mask ? p.tile_mask[tile] : 0x7ffffffu) : 1u;
    if (p.kvol < 32) mask &= (p.kvol == 32 ? 0xffffffffu : ((1u << p.kvol) - 1u));
    const int kchunks = (p.cin + BK - 1) / BK;
    const int steps = __popc(mask) * kchunks;

    // A-load mapping: 2 float4 per thread: rows (tid/4) and (tid/4 + 64), k quad tid%4
    const int a_row = tid >> 2;
    const int a_kq = tid & 3;
    // B-load mapping
    constexpr int B_F4 = BK * BN / 4;
    const int b_k = tid / (BN / 4);
    const int b_c4 = tid % (BN / 4);

    int32_t src[2] = {-1, -1};
    float4 ra[2], rb;
    int cur_o = -1;
    uint32_t mrem = mask;

    auto fetch = [&](int step) {
        const int kc = step % kchunks;
        if (kc == 0) {
            cur_o = __ffs(mrem) - 1;
            mrem &= mrem - 1;
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int64_t r = m0 + a_row + 64 * i;
                int32_t s = -1;
                if (r < p.n_out) s = p.nbr ? p.nbr[(int64_t)cur_o * p.n_out + r] : (int32_t)r;
                src[i] = s < 0 ? -1 : (s >> p.in_shift);
            }
        }
        const int k0 = kc * BK + a_kq * 4;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (src[i] >= 0 && k0 < p.cin) {
                const bool from_a = k0 < p.cin_a;
                const float* g = from_a ? p.in + (int64_t)src[i] * p.cin_a + k0
                                        : p.in_b + (int64_t)src[i] * (p.cin - p.cin_a) + (k0 - p.cin_a);
                v = *reinterpret_cast<const float4*>(g);
                if (p.flags & S3DSP_PRO_AFFINE_SILU) {
                    v.x = silu_f((v.x - p.pro_sub[k0 + 0]) * p.pro_mul[k0 + 0] + p.pro_add[k0 + 0]);
                    v.y = silu_f((v.y - p.pro_sub[k0 + 1]) * p.pro_mul[k0 + 1] + p.pro_add[k0 + 1]);
                    v.z = silu_f((v.z - p.pro_sub[k0 + 2]) * p.pro_mul[k0 + 2] + p.pro_add[k0 + 2]);
                    v.w = silu_f((v.w - p.pro_sub[k0 + 3]) * p.pro_mul[k0 + 3] + p.pro_add[k0 + 3]);
                }
            }
            ra[i] = v;
        }
        if (tid < B_F4) {
            const int k = kc * BK + b_k;  // < cin_pad (packed weights are zero padded)
            rb = *reinterpret_cast<const float4*>(p.w + ((int64_t)cur_o * p.cin_pad + k) * p.cout_pad + n0 + 4 * b_c4);
        }
    };
    auto stash = [&](int buf) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            As[buf][a_kq * 4 + 0][a_row + 64 * i] = ra[i].x;
            As[buf][a_kq * 4 + 1][a_row + 64 * i] = ra[i].y;
            As[buf][a_kq * 4 + 2][a_row + 64 * i] = ra[i].z;
            As[buf][a_kq * 4 + 3][a_row + 64 * i] = ra[i].w;
        }
        if (tid < B_F4) *reinterpret_cast<float4*>(&Bs[buf][b_k][4 * b_c4]) = rb;
    };

    const int ty = tid >> 4, tx = tid & 15;
    float acc[8][TN];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

    if (steps > 0) {
        fetch(0);
        stash(0);
        __syncthreads();
        for (int s = 0; s < steps; ++s) {
            const int buf = s & 1;
            if (s + 1 < steps) fetch(s + 1);
#pragma unroll
            for (int k = 0; k < BK; ++k) {
                const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][k][ty * 4]);
                const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][k][64 + ty * 4]);
                const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                float b[TN];
#pragma unroll
                for (int j = 0; j < TN; ++j) b[j] = Bs[buf][k][tx * TN + j];
#pragma unroll
                for (int i = 0; i < 8; ++i)
#pragma unroll
                    for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
            }
            if (s + 1 < steps) stash(buf ^ 1);
            __syncthreads();
        }
    }

    // epilogue
    const bool stats = p.gn_partials != nullptr;
    const int gs = stats ? p.cout / p.gn_groups : 1;
    double csum[TN], csq[TN];
#pragma unroll
    for (int j = 0; j < TN; ++j) csum[j] = csq[j] = 0.0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int64_t r = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
        if (r >= p.n_out) continue;
#pragma unroll
        for (int j = 0; j < TN; ++j) {
            const int col = n0 + tx * TN + j;
            if (col >= p.cout) continue;
            float v = acc[i][j] + (p.bias ? p.bias[col] : 0.f);
            if (p.residual) v += load_as_f32(p.residual, p.res_dtype, (r >> p.res_shift) * p.cout + col);
            if (stats) {
                csum[j] += (double)v;
                csq[j] += (double)v * (double)v;
            }
            if (p.flags & S3DSP_EPI_SILU) v = silu_f(v);
            if (p.flags & S3DSP_EPI_GELU) v = 0.5f * v * (1.0f + tanhf(0.7978845608028654f * (v + 0.044715f * v * v * v)));
            if (p.out_dtype == S3DSP_F32)
                reinterpret_cast<float*>(p.out)[r * p.cout + col] = v;
            else if (p.out_dtype == S3DSP_BF16)
                reinterpret_cast<__nv_bfloat16*>(p.out)[r * p.cout + col] = __float2bfloat16(v);
            else
                reinterpret_cast<__half*>(p.out)[r * p.cout + col] = __float2half(v);
        }
    }
    if (stats) {
        // deterministic: every thread's column sums to smem, then each group
        // summed over row groups and columns in a fixed order
#pragma unroll
        for (int j = 0; j < TN; ++j) {
            colsum[ty][tx * TN + j][0] = csum[j];
            colsum[ty][tx * TN + j][1] = csq[j];
        }
        __syncthreads();
        const int limit = min(BN, p.cout - n0);
        const int g_lo = n0 / gs;
        const int g_hi = min(p.gn_groups - 1, (n0 + limit - 1) / gs);
        for (int g = g_lo + tid; g <= g_hi; g += NT) {
            const int c_lo = max(g * gs - n0, 0), c_hi = min((g + 1) * gs - n0, limit);
            double a = 0.0, b = 0.0;
            for (int y = 0; y < 16; ++y)
                for (int c = c_lo; c < c_hi; ++c) {
                    a += colsum[y][c][0];
                    b += colsum[y][c][1];
                }
            // a group split across two column tiles gets exactly two adds onto a
            // zeroed slot, which is order independent
            atomicAdd(p.gn_partials + ((int64_t)tile * p.gn_groups + g) * 2 + 0, a);
            atomicAdd(p.gn_partials + ((int64_t)tile * p.gn_groups + g) * 2 + 1, b);
        }
    }
}

}  // namespace

namespace s3dsp {

cudaError_t launch_conv_f32(s3dsp_context* ctx, const s3dsp_kmap* kmap, int kvol, const float* in,
                            const float* in_b, int cin_a, int64_t n_in, int cin, int in_shift, const float* w,
                            const float* bias, const void* residual, uint32_t res_dtype,
                            int res_shift, void* out, uint32_t out_dtype, int64_t n_out, int cout,
                            uint32_t flags, const float* pro_sub, const float* pro_mul,
                            const float* pro_add, double* gn_partials, int gn_groups) {
    F32ConvParams p;
    p.in = in;
    p.in_b = in_b;
    p.cin_a = in_b ? cin_a : cin;
    p.n_in = n_in;
    p.cin = cin;
    p.in_shift = in_shift;
    p.nbr = kmap ? kmap->nbr : nullptr;
    p.tile_mask = kmap ? kmap->tile_mask : nullptr;
    p.kvol = kvol;
    p.w = w;
    p.cin_pad = (cin + BK - 1) / BK * BK;
    const int bn = (cout % 64 == 0 || cout > 64) ? 64 : 32;
    p.cout_pad = (cout + 63) / 64 * 64;
    p.bias = bias;
    p.residual = residual;
    p.res_dtype = res_dtype;
    p.res_shift = res_shift;
    p.out = out;
    p.out_dtype = out_dtype;
    p.n_out = n_out;
    p.cout = cout;
    p.flags = flags;
    p.pro_sub = pro_sub;
    p.pro_mul = pro_mul;
    p.pro_add = pro_add;
    p.gn_partials = gn_partials;
    p.gn_groups = gn_groups;
    const int64_t tiles = (n_out + BM - 1) / BM;
    if (gn_partials) {
        cudaError_t e = cudaMemsetAsync(gn_partials, 0, sizeof(double) * 2 * (size_t)gn_groups * (size_t)tiles,
                                        ctx->stream);
        if (e != cudaSuccess) return e;
    }
    const dim3 grid((unsigned)tiles, (unsigned)((cout + bn - 1) / bn));
    if (bn == 64)
        launch_pdl(conv_f32_kernel<64>, dim3(grid), dim3(NT), 0, ctx->stream, p);
    else
        launch_pdl(conv_f32_kernel<32>, dim3(grid), dim3(NT), 0, ctx->stream, p);
    return cudaGetLastError();
}

}  // namespace s3dsp
