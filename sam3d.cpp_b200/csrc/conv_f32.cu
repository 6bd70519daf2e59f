// F32-strict implicit-gather sparse convolution on the FP32 pipes.
//
// out[r, :] = sum_{o active} sum_ci pro(in[nbr_o(r) >> in_shift, ci]) * W[o, ci, :]
//             + bias (+ residual) (-> SiLU)
// One CTA owns a 128-row x BN-column output tile and walks (offset, 16-channel
// chunk) steps; gathered rows are staged through registers into shared memory
// (transposed, so each thread reads 4 consecutive rows as one float4), double
// buffered. Each thread accumulates 8 rows x BN/16 columns in registers (no
// atomics); with BN >= 64 its columns are groups of four at a stride of 64
// (4tx.., 64+4tx..), so a warp's weight reads are contiguous 16-byte loads.
// Every output sums its products in the same order (offset, then channel) for
// any BN. Offsets with no neighbour in the tile (per-tile bitmask from the
// kmap) are skipped.
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

// column of the tile held by thread tx as its j-th column
template <int BN>
__device__ __forceinline__ int f32_col(int tx, int j) {
    if constexpr (BN >= 64) return 64 * (j >> 2) + 4 * tx + (j & 3);
    else return tx * (BN / 16) + j;
}

template <int BN>
__global__ void __launch_bounds__(NT, BN >= 128 ? 2 : 1) conv_f32_kernel(const F32ConvParams p) {
    pdl_wait();
    pdl_trigger();
    constexpr int TN = BN / 16;
    // the two stages of A and B, and after the main loop the GroupNorm column sums
    constexpr int kStageBytes = 2 * BK * BM * 4 + 2 * BK * BN * 4;
    constexpr int kColBytes = 16 * BN * 2 * 8;
    __shared__ __align__(16) unsigned char smem_raw[kStageBytes > kColBytes ? kStageBytes : kColBytes];
    auto As = reinterpret_cast<float (*)[BK][BM]>(smem_raw);
    auto Bs = reinterpret_cast<float (*)[BK][BN]>(smem_raw + 2 * BK * BM * 4);
    auto colsum = reinterpret_cast<double (*)[BN][2]>(smem_raw);  // per row group ty, fixed-order sums

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
    // B-load mapping: BK x BN floats as float4s, NB4 per thread
    constexpr int B_F4 = BK * BN / 4;
    constexpr int NB4 = (B_F4 + NT - 1) / NT;

    int32_t src[2] = {-1, -1};
    float4 ra[2], rb[NB4];
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
#pragma unroll
        for (int q = 0; q < NB4; ++q) {
            const int f = tid + NT * q;
            if (f < B_F4) {
                const int k = kc * BK + f / (BN / 4);  // < cin_pad (packed weights are zero padded)
                rb[q] = *reinterpret_cast<const float4*>(p.w + ((int64_t)cur_o * p.cin_pad + k) * p.cout_pad + n0 +
                                                         4 * (f % (BN / 4)));
            }
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
#pragma unroll
        for (int q = 0; q < NB4; ++q) {
            const int f = tid + NT * q;
            if (f < B_F4) *reinterpret_cast<float4*>(&Bs[buf][f / (BN / 4)][4 * (f % (BN / 4))]) = rb[q];
        }
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
                if constexpr (BN >= 64) {
#pragma unroll
                    for (int g = 0; g < TN / 4; ++g) {
                        const float4 b4 = *reinterpret_cast<const float4*>(&Bs[buf][k][64 * g + 4 * tx]);
                        b[4 * g + 0] = b4.x;
                        b[4 * g + 1] = b4.y;
                        b[4 * g + 2] = b4.z;
                        b[4 * g + 3] = b4.w;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < TN; ++j) b[j] = Bs[buf][k][tx * TN + j];
                }
#pragma unroll
                for (int i = 0; i < 8; ++i)
#pragma unroll
                    for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
            }
            if (s + 1 < steps) stash(buf ^ 1);
            __syncthreads();
        }
    }

    // epilogue, by groups of GJ columns (GJ f64 column sums live at a time);
    // the column sums reuse the stage buffers, which the last step's barrier freed
    const bool stats = p.gn_partials != nullptr;
    const int gs = stats ? p.cout / p.gn_groups : 1;
    constexpr int GJ = TN >= 4 ? 4 : TN;
#pragma unroll
    for (int g = 0; g < TN / GJ; ++g) {
        double csum[GJ], csq[GJ];
#pragma unroll
        for (int jj = 0; jj < GJ; ++jj) csum[jj] = csq[jj] = 0.0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int64_t r = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
            if (r >= p.n_out) continue;
#pragma unroll
            for (int jj = 0; jj < GJ; ++jj) {
                const int j = g * GJ + jj;
                const int col = n0 + f32_col<BN>(tx, j);
                if (col >= p.cout) continue;
                float v = acc[i][j] + (p.bias ? p.bias[col] : 0.f);
                if (p.residual) v += load_as_f32(p.residual, p.res_dtype, (r >> p.res_shift) * p.cout + col);
                if (stats) {
                    csum[jj] += (double)v;
                    csq[jj] += (double)v * (double)v;
                }
                if (p.flags & S3DSP_EPI_SILU) v = silu_f(v);
                if (p.flags & S3DSP_EPI_GELU)
                    v = 0.5f * v * (1.0f + tanhf(0.7978845608028654f * (v + 0.044715f * v * v * v)));
                if (p.out_dtype == S3DSP_F32)
                    reinterpret_cast<float*>(p.out)[r * p.cout + col] = v;
                else if (p.out_dtype == S3DSP_BF16)
                    reinterpret_cast<__nv_bfloat16*>(p.out)[r * p.cout + col] = __float2bfloat16(v);
                else
                    reinterpret_cast<__half*>(p.out)[r * p.cout + col] = __float2half(v);
            }
        }
        if (stats) {
#pragma unroll
            for (int jj = 0; jj < GJ; ++jj) {
                colsum[ty][f32_col<BN>(tx, g * GJ + jj)][0] = csum[jj];
                colsum[ty][f32_col<BN>(tx, g * GJ + jj)][1] = csq[jj];
            }
        }
    }
    if (stats) {
        // deterministic: each group summed over row groups and columns in a fixed order
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
    p.cout_pad = (cout + 63) / 64 * 64;
    // 128-column tiles (8 x 8 outputs per thread) for layers of at least two
    // such blocks: on B200, config 2 (C = 256) 1.56 vs 1.70 ms per conv; at
    // C = 128 the halved CTA count made them slower (0.56 vs 0.46 ms)
    const int bn = p.cout_pad % 256 == 0 ? 128 : (cout % 64 == 0 || cout > 64) ? 64 : 32;
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
    if (bn == 128)
        launch_pdl(conv_f32_kernel<128>, dim3(grid), dim3(NT), 0, ctx->stream, p);
    else if (bn == 64)
        launch_pdl(conv_f32_kernel<64>, dim3(grid), dim3(NT), 0, ctx->stream, p);
    else
        launch_pdl(conv_f32_kernel<32>, dim3(grid), dim3(NT), 0, ctx->stream, p);
    return cudaGetLastError();
}

}  // namespace s3dsp
