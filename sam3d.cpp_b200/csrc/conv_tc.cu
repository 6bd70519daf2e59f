// K3 (BF16) implicit-gather sparse convolution on the 5th-generation tensor
// cores: tcgen05.mma with the f32 accumulator in TMEM.
//
// Tile: 128 output rows x BN output channels per CTA (BN = a multiple of 16,
// <= 256). The reduction walks (active offset, 64-channel chunk) steps. Per
// step, stage s of a multi-stage shared-memory ring receives
//   A: the 128 gathered input rows (64 bf16 = 128 B each) by cp.async from
//      the gather index (16-byte copies, zero-filled for missing neighbours),
//      written in the 128-byte-swizzled K-major layout the MMA descriptor
//      expects;
//   B: the BN x 64 weight tile W[o][n0:n0+BN][k0:k0+64] by one TMA tensor
//      load (128-byte swizzle), no multicast.
// One elected thread issues 4 tcgen05.mma (M=128, N=BN, K=16) per step and
// releases the stage with tcgen05.commit. The epilogue warps read the
// accumulator back with tcgen05.ld, add bias / residual, optionally SiLU,
// accumulate GroupNorm partial sums and store; nothing is accumulated
// through atomics on the output.
//
// Warp roles (192 threads): warps 0-3 gather A and then run the epilogue
// (warp w owns TMEM lanes 32w..32w+31 = tile rows); warp 4 issues the weight
// TMA; warp 5 owns the TMEM allocation and issues the MMAs.
//
// Every mbarrier wait is bounded (about two seconds of %globaltimer); on
// timeout the CTA records kErrPipelineTimeout, stops issuing work and exits
// through the common teardown, which frees its TMEM.
//
// Replaces the GGML get_rows + mul_mat chains of slat_flow_graph.cpp:112-155
// (SLat conv) and mesh_decoder_graph.cpp:81-103 (mesh conv, per-offset form)
// as one gather-GEMM; in_shift = 3 gathers the parent row of a child, which
// is repeat_children (mesh_decoder_graph.cpp:32-38) without materialising it.
#include "s3dsp_internal.h"

#include <cudaTypedefs.h>

using namespace s3dsp;

namespace {

constexpr int kThreads = 192;
constexpr int kAStage = 128 * 128;  // bytes: 128 rows x 64 bf16
constexpr int kLag = 2;             // cp.async groups kept in flight per producer thread
constexpr int kMaxKvol = 27;
constexpr unsigned long long kWaitNs = 2000000000ull;  // 2 s

struct TcParams {
    const __nv_bfloat16* in;
    int cin;
    int in_shift;
    const int32_t* nbr;         // [kvol][n_out] or null (identity)
    const uint32_t* tile_mask;  // [tiles] or null
    int kvol;
    int cout_pad;               // packed weight rows per offset
    int bn;
    int stages;
    uint32_t idesc;
    const float* bias;
    const void* residual;
    uint32_t res_dtype;
    int res_shift;
    void* out;
    uint32_t out_dtype;
    int64_t n_out;
    int cout;
    uint32_t flags;
    double* gn_partials;
    int gn_groups;
    uint32_t* status;
};

// ---------------------------------------------------------------------------
// PTX helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait. Returns false (and raises the CTA abort flag) on timeout or
// when another role already aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          uint32_t* status) {
    if (mbar_try(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try(bar, parity)) return true;
        if ((it & 255u) == 0) {
            if (*abort_flag) return false;
            if (global_ns() - t0 > kWaitNs) {
                *abort_flag = 1;
                atomicOr(status, kErrPipelineTimeout);
                return false;
            }
        }
    }
}
__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"((unsigned long long)map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major operand in the 128-byte swizzle canonical layout: rows of 128 B,
// 8-row (1024 B) swizzle atoms stacked along M/N (stride byte offset 1024),
// descriptor version 1, layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
    return (uint64_t)((addr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + __expf(-v)); }

__device__ __forceinline__ float load_as_f32(const void* p, uint32_t dt, int64_t i) {
    if (dt == S3DSP_F32) return reinterpret_cast<const float*>(p)[i];
    if (dt == S3DSP_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    return __half2float(reinterpret_cast<const __half*>(p)[i]);
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads, 1)
    conv_tc_kernel(const TcParams p, const __grid_constant__ CUtensorMap wmap) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte aligned base for the swizzled tiles
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int S = p.stages;
    const int bstage = p.bn * 128;
    uint8_t* sA = smem;
    uint8_t* sB = smem + (size_t)S * kAStage;
    uint64_t* full = reinterpret_cast<uint64_t*>(sB + (size_t)S * bstage);
    uint64_t* empty = full + S;
    uint64_t* accum = empty + S;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(accum + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
    double* gsum = reinterpret_cast<double*>(tmem_holder + 4);           // [64][2]
    int32_t* sidx = reinterpret_cast<int32_t*>(gsum + 128);              // [kvol][128]

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int tile = blockIdx.x;
    const int64_t m0 = (int64_t)tile * 128;
    const int n0 = blockIdx.y * p.bn;

    uint32_t mask = p.nbr ? (p.tile_mask ? p.tile_mask[tile] : 0x7ffffffu) : 1u;
    mask &= (p.kvol >= 32) ? 0xffffffffu : ((1u << p.kvol) - 1u);
    const int kchunks = (p.cin + 63) / 64;
    const int T = __popc(mask) * kchunks;
    const uint32_t tcols = p.bn <= 32 ? 32u : (p.bn <= 64 ? 64u : (p.bn <= 128 ? 128u : 256u));

    // ---- setup: barriers, TMEM, gather indices ----
    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(smem_u32(full + s), 128 + 1);
            mbar_init(smem_u32(empty + s), 1);
        }
        mbar_init(smem_u32(accum), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 5) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                     "r"(tcols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (p.gn_partials)
        for (int i = tid; i < 128; i += kThreads) gsum[i] = 0.0;
    // gather indices of the active offsets for the tile's 128 rows
    for (int i = tid; i < kMaxKvol * 128; i += kThreads) {
        const int o = i >> 7, row = i & 127;
        if (!((mask >> o) & 1u)) continue;
        const int64_t r = m0 + row;
        int32_t s = -1;
        if (r < p.n_out) s = p.nbr ? __ldg(p.nbr + (int64_t)o * p.n_out + r) : (int32_t)r;
        sidx[i] = s < 0 ? -1 : (s >> p.in_shift);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp < 4) {
        // ================= A producers: gathered rows via cp.async =================
        const int c16 = tid & 7;  // 16-byte chunk within a 128-byte row
        const int rg = tid >> 3;  // rows rg + 16*i
        uint32_t mrem = mask;
        int o = 0;
        bool ok = true;
        for (int it = 0; it < T; ++it) {
            const int s = it % S;
            const uint32_t ph = (uint32_t)(it / S) & 1u;
            const int kc = it % kchunks;
            if (kc == 0) {
                o = __ffs(mrem) - 1;
                mrem &= mrem - 1;
            }
            if (!mbar_wait(smem_u32(empty + s), ph ^ 1u, abort_flag, p.status)) {
                ok = false;
                break;
            }
            const int k0 = kc * 64 + c16 * 8;
            const uint32_t a_base = smem_u32(sA + (size_t)s * kAStage);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int row = rg + 16 * i;
                const int32_t src = sidx[o * 128 + row];
                const bool valid = src >= 0 && k0 < p.cin;
                const void* g = valid ? (const void*)(p.in + (int64_t)src * p.cin + k0) : (const void*)p.in;
                cp_async_16(a_base + row * 128 + ((c16 ^ (row & 7)) << 4), g, valid ? 16u : 0u);
            }
            cp_async_commit();
            if (it >= kLag) {
                cp_async_wait<kLag>();
                fence_proxy_async();
                mbar_arrive(smem_u32(full + (it - kLag) % S));
            }
        }
        cp_async_wait<0>();
        fence_proxy_async();
        if (ok)
            for (int it = (T > kLag ? T - kLag : 0); it < T; ++it) mbar_arrive(smem_u32(full + it % S));

        // ================= epilogue =================
        const int row = warp * 32 + lane;
        const int64_t r = m0 + row;
        const bool have_acc = T > 0 && ok && mbar_wait(smem_u32(accum), 0, abort_flag, p.status);
        tc_fence_after();
        const bool stats = p.gn_partials != nullptr;
        const int gs = stats ? p.cout / p.gn_groups : 1;
        const bool row_ok = r < p.n_out;
        const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16);
        for (int c0 = 0; c0 < p.bn; c0 += 16) {
            uint32_t v[16];
            if (have_acc) {
                tmem_ld16(taddr + (uint32_t)c0, v);
            } else {
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = 0u;
            }
            float f[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int col = n0 + c0 + j;
                float x = __uint_as_float(v[j]);
                if (col < p.cout) {
                    if (p.bias) x += __ldg(p.bias + col);
                    if (p.residual && row_ok)
                        x += load_as_f32(p.residual, p.res_dtype, (r >> p.res_shift) * p.cout + col);
                }
                f[j] = x;
            }
            if (stats) {
                // columns are warp-uniform, so group changes are too
                double s1 = 0.0, s2 = 0.0;
                int g_cur = -1;
                for (int j = 0; j <= 16; ++j) {
                    const int col = n0 + c0 + j;
                    const int g = (j < 16 && col < p.cout) ? col / gs : -2;
                    if (g != g_cur) {
                        if (g_cur >= 0) {
#pragma unroll
                            for (int d = 16; d > 0; d >>= 1) {
                                s1 += __shfl_xor_sync(0xffffffffu, s1, d);
                                s2 += __shfl_xor_sync(0xffffffffu, s2, d);
                            }
                            if (lane == 0) {
                                atomicAdd(gsum + 2 * g_cur, s1);
                                atomicAdd(gsum + 2 * g_cur + 1, s2);
                            }
                        }
                        s1 = s2 = 0.0;
                        g_cur = g;
                    }
                    if (g >= 0 && row_ok) {
                        s1 += (double)f[j];
                        s2 += (double)f[j] * (double)f[j];
                    }
                }
            }
            if (p.flags & S3DSP_EPI_SILU) {
#pragma unroll
                for (int j = 0; j < 16; ++j) f[j] = silu_f(f[j]);
            }
            if (row_ok) {
                const int nvalid = min(16, p.cout - (n0 + c0));
                if (p.out_dtype == S3DSP_F32) {
                    float* dst = reinterpret_cast<float*>(p.out) + r * p.cout + n0 + c0;
                    if (nvalid == 16 && (p.cout & 3) == 0) {
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            reinterpret_cast<float4*>(dst)[q] = make_float4(f[4 * q], f[4 * q + 1], f[4 * q + 2], f[4 * q + 3]);
                    } else {
                        for (int j = 0; j < nvalid; ++j) dst[j] = f[j];
                    }
                } else {
                    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.out) + r * p.cout + n0 + c0;
                    if (p.out_dtype == S3DSP_BF16 && nvalid == 16 && (p.cout & 7) == 0) {
                        uint32_t w[8];
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            const __nv_bfloat162 h2 = __floats2bfloat162_rn(f[2 * q], f[2 * q + 1]);
                            w[q] = *reinterpret_cast<const uint32_t*>(&h2);
                        }
                        reinterpret_cast<uint4*>(dst)[0] = make_uint4(w[0], w[1], w[2], w[3]);
                        reinterpret_cast<uint4*>(dst)[1] = make_uint4(w[4], w[5], w[6], w[7]);
                    } else if (p.out_dtype == S3DSP_BF16) {
                        for (int j = 0; j < nvalid; ++j) dst[j] = __float2bfloat16(f[j]);
                    } else {
                        __half* hd = reinterpret_cast<__half*>(p.out) + r * p.cout + n0 + c0;
                        for (int j = 0; j < nvalid; ++j) hd[j] = __float2half(f[j]);
                    }
                }
            }
        }
        if (stats) {
            asm volatile("bar.sync 1, 128;" ::: "memory");
            const int g_lo = n0 / gs;
            const int g_hi = min(p.gn_groups - 1, (min(n0 + p.bn, p.cout) - 1) / gs);
            for (int g = g_lo + tid; g <= g_hi; g += 128) {
                atomicAdd(p.gn_partials + ((int64_t)tile * p.gn_groups + g) * 2 + 0, gsum[2 * g]);
                atomicAdd(p.gn_partials + ((int64_t)tile * p.gn_groups + g) * 2 + 1, gsum[2 * g + 1]);
            }
        }
        tc_fence_before();
    } else if (warp == 4) {
        // ================= B producer: weight tiles via TMA =================
        if (lane == 0) {
            uint32_t mrem = mask;
            int o = 0;
            const uint32_t bytes = (uint32_t)bstage;
            for (int it = 0; it < T; ++it) {
                const int s = it % S;
                const uint32_t ph = (uint32_t)(it / S) & 1u;
                const int kc = it % kchunks;
                if (kc == 0) {
                    o = __ffs(mrem) - 1;
                    mrem &= mrem - 1;
                }
                if (!mbar_wait(smem_u32(empty + s), ph ^ 1u, abort_flag, p.status)) break;
                const uint32_t fb = smem_u32(full + s);
                mbar_arrive_tx(fb, bytes);
                tma_load_2d(smem_u32(sB + (size_t)s * bstage), &wmap, kc * 64, o * p.cout_pad + n0, fb);
            }
        }
    } else {
        // ================= MMA issuer =================
        if (lane == 0) {
            bool ok = true;
            for (int it = 0; it < T; ++it) {
                const int s = it % S;
                const uint32_t ph = (uint32_t)(it / S) & 1u;
                if (!mbar_wait(smem_u32(full + s), ph, abort_flag, p.status)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a0 = smem_u32(sA + (size_t)s * kAStage);
                const uint32_t b0 = smem_u32(sB + (size_t)s * bstage);
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    mma_bf16(tmem, sw128_desc(a0 + 32 * k), sw128_desc(b0 + 32 * k), p.idesc,
                             (it > 0 || k > 0) ? 1u : 0u);
                mma_commit(smem_u32(empty + s));
            }
            if (ok && T > 0) mma_commit(smem_u32(accum));
        }
        __syncwarp();
    }

    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tcols) : "memory");
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
    return fn;
}

size_t smem_bytes(int stages, int bn) {
    return 1024 /*align slack*/ + (size_t)stages * (kAStage + bn * 128) + (2 * stages + 1) * 8 + 16 +
           128 * 8 /*gsum*/ + kMaxKvol * 128 * 4 /*sidx*/;
}

}  // namespace

namespace s3dsp {

int tc_pick_bn(int cout) {
    const int cp = (cout + 15) / 16 * 16;
    if (cp <= 256) return cp;
    for (int bn = 256; bn >= 16; bn -= 16)
        if (cp % bn == 0) return bn;
    return 16;
}

cudaError_t launch_conv_tc(s3dsp_context* ctx, const s3dsp_kmap* kmap, int kvol,
                           const __nv_bfloat16* in, int64_t n_in, int cin, int in_shift,
                           const __nv_bfloat16* w, const float* bias, const void* residual,
                           uint32_t res_dtype, int res_shift, void* out, uint32_t out_dtype,
                           int64_t n_out, int cout, uint32_t flags, double* gn_partials,
                           int gn_groups, char* error, uint64_t error_capacity, s3d_status* st) {
    (void)n_in;
    *st = S3D_OK;
    const int cout_pad = (cout + 15) / 16 * 16;
    const int cin_pad = (cin + 63) / 64 * 64;
    const int bn = tc_pick_bn(cout);
    int stages = (int)((200 * 1024) / (kAStage + bn * 128));
    if (stages > 8) stages = 8;
    if (stages < kLag + 1) stages = kLag + 1;

    auto encode = get_encode_fn();
    if (!encode) {
        *st = fail(error, error_capacity, S3D_INTERNAL_ERROR, "cuTensorMapEncodeTiled unavailable");
        return cudaErrorNotSupported;
    }
    CUtensorMap map;
    const cuuint64_t dims[2] = {(cuuint64_t)cin_pad, (cuuint64_t)kvol * (cuuint64_t)cout_pad};
    const cuuint64_t strides[1] = {(cuuint64_t)cin_pad * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)bn};
    const cuuint32_t estr[2] = {1, 1};
    CUresult cr = encode(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (void*)w, dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) {
        *st = fail(error, error_capacity, S3D_INTERNAL_ERROR, "cuTensorMapEncodeTiled failed (%d)", (int)cr);
        return cudaErrorInvalidValue;
    }
    TcParams p;
    p.in = in;
    p.cin = cin;
    p.in_shift = in_shift;
    p.nbr = kmap ? kmap->nbr : nullptr;
    p.tile_mask = kmap ? kmap->tile_mask : nullptr;
    p.kvol = kvol;
    p.cout_pad = cout_pad;
    p.bn = bn;
    p.stages = stages;
    p.idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(bn >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
    p.bias = bias;
    p.residual = residual;
    p.res_dtype = res_dtype;
    p.res_shift = res_shift;
    p.out = out;
    p.out_dtype = out_dtype;
    p.n_out = n_out;
    p.cout = cout;
    p.flags = flags;
    p.gn_partials = gn_partials;
    p.gn_groups = gn_groups;
    p.status = ctx->d_status;

    const size_t smem = smem_bytes(stages, bn);
    cudaError_t e = cudaFuncSetAttribute(conv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const int64_t tiles = (n_out + 127) / 128;
    if (gn_partials) {
        e = cudaMemsetAsync(gn_partials, 0, sizeof(double) * 2 * (size_t)gn_groups * (size_t)tiles, ctx->stream);
        if (e != cudaSuccess) return e;
    }
    const dim3 grid((unsigned)tiles, (unsigned)(cout_pad / bn));
    conv_tc_kernel<<<grid, kThreads, smem, ctx->stream>>>(p, map);
    (void)cin_pad;
    return cudaGetLastError();
}

}  // namespace s3dsp
