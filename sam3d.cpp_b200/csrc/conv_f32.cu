// F32-strict implicit-gather sparse convolution on the FP32 pipes.
//
// out[r, :] = sum_{o active} sum_ci pro(in[nbr_o(r) >> in_shift, ci]) * W[o, ci, :]
//             + bias (+ residual) (-> SiLU)
// One CTA owns a 128-row x BN-column output tile and walks (offset, 16-channel
// chunk) steps. Each thread accumulates 8 rows x BN/16 columns in registers
// (no atomics); with BN >= 64 its columns are groups of four at a stride of
// 64 (4tx.., 64+4tx..), so a warp's weight reads are contiguous 16-byte
// loads. Every output sums its products in the same order (offset, then
// channel) in both kernels, so they give the same bits. Offsets with no
// neighbour in the tile (per-tile bitmask from the kmap) are skipped.
//  * conv_f32_ms_kernel (BN = 64 or 128, every wider layer): rows and weights
//    go to a 4-stage shared-memory ring by cp.async, and the inner loop runs
//    packed two-lane FP32 FMAs (fma.rn.f32x2). On B200 it is 5-11 % faster
//    than the register-staged form on the 64^3-128^3 shells at C = 64-256.
//  * conv_f32_kernel (BN = 32, layers of at most 32 channels): gathered rows
//    staged through registers into shared memory (transposed), double buffered.
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

// Epilogue of a 128 x BN tile held as acc[8][BN / 16] per thread (thread
// (ty, tx): rows 4ty.. and 64 + 4ty.., columns f32_col<BN>(tx, j)): bias,
// residual, GroupNorm column sums (f64, by groups of GJ columns: GJ sums live
// at a time), SiLU / GELU and the store; then the tile's GroupNorm partials
// from the per-row-group column sums in a fixed order. `colsum` may alias the
// main loop's shared memory once every thread is past its last read of it.
template <int BN>
__device__ __forceinline__ void f32_epilogue(const F32ConvParams& p, const float (&acc)[8][BN / 16],
                                             double (*colsum)[BN][2], int64_t m0, int n0, int tile, int tid) {
    constexpr int TN = BN / 16;
    const int ty = tid >> 4, tx = tid & 15;
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

    // the column sums reuse the stage buffers, which the last step's barrier freed
    f32_epilogue<BN>(p, acc, reinterpret_cast<double(*)[BN][2]>(smem_raw), m0, n0, tile, tid);
}


// Multistage form (BN = 64 or 128): the gathered rows and the weight rows go
// straight from global to shared memory by 16-byte cp.async, kStages deep
// (no register staging, so no load latency in the compute loop and no
// transposed stores); A rows are kept row-major with a 20-float stride and
// read as float4 along k (two distinct 16-byte addresses per warp access, in
// different bank halves). The products of every output are summed in the same
// order as in conv_f32_kernel, so both give the same bits.
constexpr int kStages = 4;
constexpr int kAPad = BK + 4;  // floats per A row in shared memory (80 bytes)

// 16-byte copy, or 16 zero bytes (nothing is read; `base` only keeps the
// source operand a valid address)
__device__ __forceinline__ void cp16(float* dst, const float* src, bool valid, const float* base) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(valid ? src : base), "r"(valid ? 16u : 0u)
                 : "memory");
}

template <int BN>
constexpr int ms_stage_floats() { return BM * kAPad + BK * BN; }
template <int BN>
constexpr int ms_smem_bytes() {
    return kStages * ms_stage_floats<BN>() * 4 > 16 * BN * 16 ? kStages * ms_stage_floats<BN>() * 4 : 16 * BN * 16;
}

template <int BN>
__global__ void __launch_bounds__(NT, 2) conv_f32_ms_kernel(const F32ConvParams p) {
    pdl_wait();
    pdl_trigger();
    constexpr int TN = BN / 16;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float* sm = reinterpret_cast<float*>(smem_raw);

    const int tid = threadIdx.x;
    const int64_t m0 = (int64_t)blockIdx.x * BM;
    const int n0 = blockIdx.y * BN;
    const int tile = blockIdx.x;

    uint32_t mask = p.nbr ? (p.tile_mask ? p.tile_mask[tile] : 0x7ffffffu) : 1u;
    if (p.kvol < 32) mask &= (1u << p.kvol) - 1u;
    const int kchunks = (p.cin + BK - 1) / BK;
    const int steps = __popc(mask) * kchunks;
    const bool pro = (p.flags & S3DSP_PRO_AFFINE_SILU) != 0;

    // issue side: this thread's A chunks are rows a_row, a_row + 64, 4-float quad a_kq
    const int a_row = tid >> 2;
    const int a_kq = tid & 3;
    constexpr int B_F4 = BK * BN / 4;
    constexpr int NB4 = (B_F4 + NT - 1) / NT;
    uint32_t mrem = mask;
    int iss_o = -1;
    int32_t src[2] = {-1, -1}, nxt[2] = {-1, -1};
    auto load_src = [&](int o, int32_t (&dst)[2]) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int64_t r = m0 + a_row + 64 * i;
            int32_t v = -1;
            if (r < p.n_out) v = p.nbr ? __ldg(p.nbr + (int64_t)o * p.n_out + r) : (int32_t)r;
            dst[i] = v < 0 ? -1 : (v >> p.in_shift);
        }
    };
    int nxt_o = -1;
    if (mrem) {
        nxt_o = __ffs(mrem) - 1;
        mrem &= mrem - 1;
        load_src(nxt_o, nxt);
    }
    uint32_t vbits = 0;  // validity of this thread's two A chunks, two bits per issued stage
    auto issue = [&](int j) {
        const int kc = j % kchunks;
        if (kc == 0) {  // next offset: its entries were loaded one offset ago
            iss_o = nxt_o;
            src[0] = nxt[0];
            src[1] = nxt[1];
            if (mrem) {
                nxt_o = __ffs(mrem) - 1;
                mrem &= mrem - 1;
                load_src(nxt_o, nxt);
            }
        }
        float* As = sm + (j % kStages) * ms_stage_floats<BN>();
        float* Bs = As + BM * kAPad;
        const int k0 = kc * BK + a_kq * 4;
        uint32_t v2 = 0;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const bool valid = src[i] >= 0 && k0 < p.cin;
            const bool from_a = k0 < p.cin_a;
            const float* g = from_a ? p.in + (int64_t)src[i] * p.cin_a + k0
                                    : p.in_b + (int64_t)src[i] * (p.cin - p.cin_a) + (k0 - p.cin_a);
            cp16(As + (a_row + 64 * i) * kAPad + a_kq * 4, g, valid, p.in);
            v2 |= (uint32_t)valid << i;
        }
        vbits = (vbits << 2) | v2;
#pragma unroll
        for (int q = 0; q < NB4; ++q) {
            const int f = tid + NT * q;
            if (f < B_F4) {
                const int kr = f / (BN / 4), c4 = f % (BN / 4);
                cp16(Bs + kr * BN + 4 * c4,
                     p.w + ((int64_t)iss_o * p.cin_pad + kc * BK + kr) * p.cout_pad + n0 + 4 * c4, true, p.w);
            }
        }
    };

    const int ty = tid >> 4, tx = tid & 15;
    float acc[8][TN];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

#pragma unroll
    for (int j = 0; j < kStages - 1; ++j) {
        if (j < steps) issue(j);
        else vbits <<= 2;
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    for (int s = 0; s < steps; ++s) {
        asm volatile("cp.async.wait_group %0;" ::"n"(kStages - 2) : "memory");
        __syncthreads();  // stage s landed everywhere; stage s - 1 is free for the refill below
        if (s + kStages - 1 < steps) issue(s + kStages - 1);
        else vbits <<= 2;
        asm volatile("cp.async.commit_group;" ::: "memory");
        const float* As = sm + (s % kStages) * ms_stage_floats<BN>();
        const float* Bs = As + BM * kAPad;
        if (pro) {
            // GroupNorm + SiLU of the previous layer on this thread's landed rows;
            // missing neighbours stay zero (the reference's mask multiply)
            const uint32_t vb = vbits >> (2 * (kStages - 1));
            const int k0 = (s % kchunks) * BK + a_kq * 4;
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                if (!((vb >> i) & 1u)) continue;
                float4* v4 = reinterpret_cast<float4*>(const_cast<float*>(As) + (a_row + 64 * i) * kAPad + a_kq * 4);
                float4 v = *v4;
                v.x = silu_f((v.x - p.pro_sub[k0 + 0]) * p.pro_mul[k0 + 0] + p.pro_add[k0 + 0]);
                v.y = silu_f((v.y - p.pro_sub[k0 + 1]) * p.pro_mul[k0 + 1] + p.pro_add[k0 + 1]);
                v.z = silu_f((v.z - p.pro_sub[k0 + 2]) * p.pro_mul[k0 + 2] + p.pro_add[k0 + 2]);
                v.w = silu_f((v.w - p.pro_sub[k0 + 3]) * p.pro_mul[k0 + 3] + p.pro_add[k0 + 3]);
                *v4 = v;
            }
            __syncthreads();
        }
#pragma unroll
        for (int kk = 0; kk < BK / 4; ++kk) {
            float4 a4[8];
#pragma unroll
            for (int i = 0; i < 8; ++i)
                a4[i] = *reinterpret_cast<const float4*>(As + ((i < 4 ? 4 * ty + i : 64 + 4 * ty + i - 4) * kAPad) +
                                                         4 * kk);
#pragma unroll
            for (int k4 = 0; k4 < 4; ++k4) {
                const int k = 4 * kk + k4;
                float b[TN];
#pragma unroll
                for (int g = 0; g < TN / 4; ++g) {
                    const float4 b4 = *reinterpret_cast<const float4*>(Bs + k * BN + 64 * g + 4 * tx);
                    b[4 * g + 0] = b4.x;
                    b[4 * g + 1] = b4.y;
                    b[4 * g + 2] = b4.z;
                    b[4 * g + 3] = b4.w;
                }
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float a = k4 == 0 ? a4[i].x : k4 == 1 ? a4[i].y : k4 == 2 ? a4[i].z : a4[i].w;
#pragma unroll
                    for (int j = 0; j < TN; j += 2) fma2(acc[i][j], acc[i][j + 1], a, b[j], b[j + 1]);
                }
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();  // the column sums reuse the stages
    f32_epilogue<BN>(p, acc, reinterpret_cast<double(*)[BN][2]>(smem_raw), m0, n0, tile, tid);
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
    if (bn == 128 || bn == 64) {
        static std::atomic<uint64_t> optin128{0}, optin64{0};
        const cudaError_t e = bn == 128 ? smem_optin((const void*)conv_f32_ms_kernel<128>, ctx->device, optin128)
                                        : smem_optin((const void*)conv_f32_ms_kernel<64>, ctx->device, optin64);
        if (e != cudaSuccess) return e;
        if (bn == 128)
            launch_pdl(conv_f32_ms_kernel<128>, dim3(grid), dim3(NT), (size_t)ms_smem_bytes<128>(), ctx->stream, p);
        else
            launch_pdl(conv_f32_ms_kernel<64>, dim3(grid), dim3(NT), (size_t)ms_smem_bytes<64>(), ctx->stream, p);
    } else
        launch_pdl(conv_f32_kernel<32>, dim3(grid), dim3(NT), 0, ctx->stream, p);
    return cudaGetLastError();
}

}  // namespace s3dsp
