// Device helpers shared by the tcgen05 convolution kernels: mbarriers with
// bounded waits, TMA and cp.async copies, tcgen05 MMA / commit / TMEM loads,
// and the typed, vectorised epilogue write-out (bias, residual, GroupNorm
// partial sums, SiLU).
#pragma once

#include "s3dsp_internal.h"

#include <cudaTypedefs.h>

#include <type_traits>

namespace s3dsp {
namespace tc {

constexpr unsigned long long kWaitNs = 2000000000ull;  // bounded mbarrier wait: 2 s

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
// --- clusters: rank, peer shared-memory addresses, the all-thread cluster barrier ---
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// shared::cluster address of the same smem variable in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
    uint32_t out;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(addr), "r"(rank));
    return out;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// 16-byte store into shared memory of a CTA of the cluster (address from map_to_rank)
__device__ __forceinline__ void st_cluster_v4(uint32_t cluster_addr, float a, float b, float c, float d) {
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(cluster_addr), "f"(a), "f"(b), "f"(c),
                 "f"(d)
                 : "memory");
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
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
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"((unsigned long long)map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
// L2 prefetch of this CTA's share of a constant tensor (the packed weights):
// CTA `i` of `n` takes bytes [i * chunk, (i + 1) * chunk), chunk a multiple of
// 16 (bytes and the base must be 16-byte multiples). A cache hint only, so it
// may run before griddepcontrol.wait: it reads nothing the kernel consumes.
__device__ __forceinline__ void prefetch_share_l2(const void* base, uint64_t bytes, uint32_t i, uint32_t n) {
    const uint64_t chunk = (bytes / n + 15) / 16 * 16;
    const uint64_t b0 = (uint64_t)i * chunk;
    if (!base || b0 >= bytes) return;
    const uint64_t len = bytes - b0 < chunk ? bytes - b0 : chunk;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(static_cast<const char*>(base) + b0),
                 "r"((uint32_t)len)
                 : "memory");
}
// L2 prefetch of a small constant array (a bias vector): one line per lane of
// the calling warp. A hint like prefetch_share_l2.
__device__ __forceinline__ void prefetch_lines_l2(const void* p, uint64_t bytes, int lane) {
    if (!p) return;
    for (uint64_t b = (uint64_t)lane * 128; b < bytes; b += 32 * 128)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(static_cast<const char*>(p) + b));
}
__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
// arrive on `bar` once all of this thread's prior cp.async copies have landed
// (counts as one of the barrier's expected arrivals)
__device__ __forceinline__ void cp_async_arrive_noinc(uint32_t bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}

// --- CTA pairs (cluster of 2, tcgen05 cta_group::2) ---
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_cluster(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// TMA tile load into this CTA's smem whose completion is counted on `bar`,
// which may be the pair leader's barrier (shared::cluster address)
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"((unsigned long long)map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void mma_bf16_pair(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
// arrive on `bar` (shared::cluster address, this CTA's or the peer's) when
// all prior pair MMAs of this thread complete
__device__ __forceinline__ void mma_commit_pair(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// bounded wait with cluster-scope acquire (arrivals released by the peer CTA)
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                                  uint32_t* status) {
    if (mbar_try_cluster(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_cluster(bar, parity)) return true;
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

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major operand in the 128-byte swizzle canonical layout: rows of 128 B,
// 8-row (1024 B) swizzle atoms stacked along M/N (stride byte offset 1024),
// descriptor version 1, layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
    return (uint64_t)((addr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// K-major operand tile of KC bf16 per row (KC = 64: 128-byte rows, SWIZZLE_128B;
// KC = 32: 64-byte rows, SWIZZLE_64B, 8-row groups 512 bytes apart). A K=16
// step advances the start address by 32 bytes in either layout.
template <int KC>
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t addr) {
    static_assert(KC == 32 || KC == 64, "KC");
    if constexpr (KC == 64) {
        return sw128_desc(addr);
    } else {
        return (uint64_t)((addr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(512 >> 4) << 32) |
               ((uint64_t)1 << 46) | ((uint64_t)4 << 61);
    }
}
// 16-byte chunk index XOR of the matching swizzle for row `row`
template <int KC>
__device__ __forceinline__ int kmajor_swz(int row) {
    if constexpr (KC == 64) return row & 7;
    else return (row >> 1) & 3;
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
// D (f32, TMEM) += A * B with A, B read as TF32 (the top 19 bits of f32 words)
__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&f)[16]) {
    uint32_t v[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int j = 0; j < 16; ++j) f[j] = __uint_as_float(v[j]);
}

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + __expf(-v)); }
// GELU, tanh form (the approximation ggml_gelu evaluates)
__device__ __forceinline__ float gelu_f(float v) {
    return 0.5f * v * (1.0f + tanhf(0.7978845608028654f * (v + 0.044715f * v * v * v)));
}

__device__ __forceinline__ float load1(const void* p, uint32_t dt, int64_t i) {
    if (dt == S3DSP_F32) return reinterpret_cast<const float*>(p)[i];
    if (dt == S3DSP_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    return __half2float(reinterpret_cast<const __half*>(p)[i]);
}
__device__ __forceinline__ void store1(void* p, uint32_t dt, int64_t i, float v) {
    if (dt == S3DSP_F32)
        reinterpret_cast<float*>(p)[i] = v;
    else if (dt == S3DSP_BF16)
        reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16(v);
    else
        reinterpret_cast<__half*>(p)[i] = __float2half(v);
}


// ---------------------------------------------------------------------------
// epilogue write-out: typed vector access, one compact loop per variant
// ---------------------------------------------------------------------------
struct NoRes {};
template <typename T>
struct Vec4;
template <>
struct Vec4<float> {
    static __device__ __forceinline__ float4 load(const void* base, int64_t i) {
        return __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + i));
    }
    static __device__ __forceinline__ void store(void* base, int64_t i, float4 v) {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(base) + i) = v;
    }
};
template <>
struct Vec4<__nv_bfloat16> {
    static __device__ __forceinline__ float4 load(const void* base, int64_t i) {
        const uint2 u = __ldg(reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(base) + i));
        const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
        const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
        return make_float4(a.x, a.y, b.x, b.y);
    }
    static __device__ __forceinline__ void store(void* base, int64_t i, float4 v) {
        const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
        *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(base) + i) =
            make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
    }
};

// Per-warp GroupNorm column sums -> colw[lc][2] (this warp's row of the
// column-sum table; columns past `limit` get zeros).
__device__ __forceinline__ void store_colsums(double* colw, int bn, int lane, int limit, const double (&s1)[2][4],
                                              const double (&s2)[2][4]) {
#pragma unroll
    for (int q = 0; q < 2; ++q)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int lc = 128 * q + 4 * lane + j;
            if (lc < bn) {
                colw[lc * 2 + 0] = lc < limit ? s1[q][j] : 0.0;
                colw[lc * 2 + 1] = lc < limit ? s2[q][j] : 0.0;
            }
        }
}

// GroupNorm partial sums (sum, sum of squares) of one 128-row tile from the
// per-warp column sums colp[kWarps][bn] (f64 pairs, left by the write-out):
// pass 1, one thread per column, sums that column over the warps in warp
// order and leaves the total in warp 0's row (each column is read and
// written by its own thread only); after `bar`, pass 2, one thread per
// group, sums the group's columns in column order into its slot. Fixed
// orders: the same result on every run. `store`: the column block holds
// whole groups, the slot is written; else a group split across two column
// blocks gets exactly two adds onto a zeroed slot (order independent).
// Lanes read consecutive 16-byte pairs in pass 1 (no bank conflicts).
template <int kWarps, int kThreads, typename Bar>
__device__ __forceinline__ void gn_tile_partials(double* colp, int bn, int n0, int limit, int gs, int groups, int tid,
                                                 double* slots, bool store, Bar bar) {
    double2* col2 = reinterpret_cast<double2*>(colp);
    for (int c = tid; c < limit; c += kThreads) {
        double a = 0.0, b = 0.0;
#pragma unroll 4
        for (int w = 0; w < kWarps; ++w) {
            const double2 v = col2[(size_t)w * bn + c];
            a += v.x;
            b += v.y;
        }
        col2[c] = make_double2(a, b);
    }
    bar();
    const int g_lo = n0 / gs;
    const int g_hi = min(groups - 1, (n0 + limit - 1) / gs);
    for (int g = g_lo + tid; g <= g_hi; g += kThreads) {
        const int c_lo = max(g * gs - n0, 0), c_hi = min((g + 1) * gs - n0, limit);
        double a = 0.0, b = 0.0;
        for (int c = c_lo; c < c_hi; ++c) {
            const double2 v = col2[c];
            a += v.x;
            b += v.y;
        }
        double* slot = slots + (size_t)g * 2;
        if (store) {
            slot[0] = a;
            slot[1] = b;
        } else {
            atomicAdd(slot + 0, a);
            atomicAdd(slot + 1, b);
        }
    }
}

// Rows lane_base .. lane_base+nrows-1 of the staged f32 tile -> global, four
// consecutive columns per lane (cout % 4 == 0, so a lane's four columns are
// all valid or all past `limit`). STATS: the warp's per-column sums of the
// values before SiLU go to colw.
template <typename OutT, typename ResT, bool SILU, bool STATS, typename P>
__device__ __forceinline__ void writeout_fast(const P& p, uint32_t so_base, int ostride, int lane_base, int lane,
                                              int64_t m0, int n0, int limit, int nrows, const float4 (&bias4)[2],
                                              double* colw) {
    double s1[2][4], s2[2][4];
    if constexpr (STATS) {
#pragma unroll
        for (int q = 0; q < 2; ++q)
#pragma unroll
            for (int j = 0; j < 4; ++j) s1[q][j] = s2[q][j] = 0.0;
    }
#pragma unroll 2
    for (int rr = 0; rr < nrows; ++rr) {
        const int row = lane_base + rr;
        const int64_t r = m0 + row;
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const int lc = 128 * q + 4 * lane;
            if (lc >= limit) continue;
            float4 v;
            asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
                         : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                         : "r"(so_base + (uint32_t)((row * ostride + lc) * 4)));
            v.x += bias4[q].x;
            v.y += bias4[q].y;
            v.z += bias4[q].z;
            v.w += bias4[q].w;
            if constexpr (!std::is_same<ResT, NoRes>::value) {
                const float4 t = Vec4<ResT>::load(p.residual, (r >> p.res_shift) * p.cout + n0 + lc);
                v.x += t.x;
                v.y += t.y;
                v.z += t.z;
                v.w += t.w;
            }
            if constexpr (STATS) {
                s1[q][0] += (double)v.x;
                s2[q][0] += (double)v.x * v.x;
                s1[q][1] += (double)v.y;
                s2[q][1] += (double)v.y * v.y;
                s1[q][2] += (double)v.z;
                s2[q][2] += (double)v.z * v.z;
                s1[q][3] += (double)v.w;
                s2[q][3] += (double)v.w * v.w;
            }
            if constexpr (SILU) {
                v.x = silu_f(v.x);
                v.y = silu_f(v.y);
                v.z = silu_f(v.z);
                v.w = silu_f(v.w);
            }
            Vec4<OutT>::store(p.out, r * p.cout + n0 + lc, v);
        }
    }
    if constexpr (STATS) store_colsums(colw, p.bn, lane, limit, s1, s2);
}

// Any dtype / ragged width: element-wise. colw as in writeout_fast (null: no
// statistics).
template <typename P>
__device__ __forceinline__ void writeout_generic(const P& p, const float* stage_out, int ostride, int lane_base,
                                                 int lane, int64_t m0, int n0, int limit, int nrows,
                                                 const float4 (&bias4)[2], double* colw) {
    double s1[2][4], s2[2][4];
    for (int q = 0; q < 2; ++q)
        for (int j = 0; j < 4; ++j) s1[q][j] = s2[q][j] = 0.0;
    for (int rr = 0; rr < nrows; ++rr) {
        const int row = lane_base + rr;
        const int64_t r = m0 + row;
        for (int q = 0; q < 2; ++q) {
            const int lc0 = 128 * q + 4 * lane;
            for (int j = 0; j < 4; ++j) {
                const int lc = lc0 + j;
                if (lc >= limit) break;
                const int col = n0 + lc;
                const float bj = j == 0 ? bias4[q].x : j == 1 ? bias4[q].y : j == 2 ? bias4[q].z : bias4[q].w;
                float v = stage_out[(size_t)row * ostride + lc] + bj;
                if (p.residual) v += load1(p.residual, p.res_dtype, (r >> p.res_shift) * p.cout + col);
                if (colw) {
                    s1[q][j] += (double)v;
                    s2[q][j] += (double)v * v;
                }
                if (p.flags & S3DSP_EPI_SILU) v = silu_f(v);
                if (p.flags & S3DSP_EPI_GELU) v = gelu_f(v);
                store1(p.out, p.out_dtype, r * p.cout + col, v);
            }
        }
    }
    if (colw) store_colsums(colw, p.bn, lane, limit, s1, s2);
}

// Phase 2 of a 128-row tile's epilogue, run by kWarps warps after the
// accumulator was staged as f32 rows of `ostride` floats at the start of
// `smem` (phase 1): warp w writes the 128 / kWarps rows from (128 / kWarps) * w, lane l owns columns
// 4l + 128q; bias, residual (row r >> res_shift), SiLU / GELU and the
// GroupNorm column sums are applied on the way out. The f64 column-sum table
// [kWarps][bn][2] follows the staged tile. gn_slot: this tile's GroupNorm
// partials (null when the tile has no slot: a padding tile past the rows);
// p.gn_partials == null means no statistics at all. `bar` synchronises the
// kWarps warps. Uses the fields bn, cout, n_out, bias, residual, res_dtype,
// res_shift, out, out_dtype, flags, gn_partials, gn_groups and gn_store of P.
template <int kWarps, typename P, typename Bar>
__device__ __forceinline__ void tile_writeout(const P& p, uint8_t* smem, int ostride, int warp, int lane, int tid,
                                              int64_t m0, int n0, double* gn_slot, Bar bar) {
    const float* stage_out = reinterpret_cast<const float*>(smem);
    const bool stats = p.gn_partials != nullptr;
    const int gs = stats ? p.cout / p.gn_groups : 1;
    constexpr int kQ = 2;  // bn <= 256 -> at most two 128-column slabs
    const int limit = min(p.bn, p.cout - n0);  // valid columns of this tile
    float4 bias4[kQ];
#pragma unroll
    for (int q = 0; q < kQ; ++q) {
        const int col = n0 + 128 * q + 4 * lane;
        bias4[q] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (p.bias && 128 * q + 4 * lane < limit) {
            bias4[q].x = __ldg(p.bias + col + 0);
            bias4[q].y = col + 1 < p.cout ? __ldg(p.bias + col + 1) : 0.f;
            bias4[q].z = col + 2 < p.cout ? __ldg(p.bias + col + 2) : 0.f;
            bias4[q].w = col + 3 < p.cout ? __ldg(p.bias + col + 3) : 0.f;
        }
    }
    constexpr int kRowsPerWarp = 128 / kWarps;
    const int lane_base = kRowsPerWarp * warp;
    const int nrows = (int)max((int64_t)0, min((int64_t)kRowsPerWarp, p.n_out - (m0 + lane_base)));
    const uint32_t so_base = smem_u32(stage_out);
    // [kWarps][bn][2]: may run past the rings (the kernels size region 0 for it)
    double* colp = reinterpret_cast<double*>(smem + (size_t)128 * ostride * 4);
    double* colw = colp + (size_t)warp * p.bn * 2;
    // One compact loop body per (out dtype, residual dtype, SiLU, stats)
    // combination: a single generic body with every variant inlined runs
    // several times slower (instruction-cache misses).
    const int out_k = (p.cout & 3) ? -1 : p.out_dtype == S3DSP_F32 ? 0 : p.out_dtype == S3DSP_BF16 ? 1 : -1;
    const int res_k = !p.residual ? 0 : p.res_dtype == S3DSP_F32 ? 1 : p.res_dtype == S3DSP_BF16 ? 2 : -1;
    const int silu_k = (p.flags & S3DSP_EPI_SILU) ? 1 : 0;
    const int sel = (out_k < 0 || res_k < 0 || (p.flags & S3DSP_EPI_GELU))
                        ? -1
                        : ((out_k * 3 + res_k) * 2 + silu_k) * 2 + (stats ? 1 : 0);
    switch (sel) {
#define S3DSP_WO(idx, OT, RT, SL, ST)                                                                        \
    case idx:                                                                                                \
        writeout_fast<OT, RT, SL, ST>(p, so_base, ostride, lane_base, lane, m0, n0, limit, nrows, bias4, colw); \
        break;
        S3DSP_WO(0, float, NoRes, false, false)
        S3DSP_WO(1, float, NoRes, false, true)
        S3DSP_WO(2, float, NoRes, true, false)
        S3DSP_WO(3, float, NoRes, true, true)
        S3DSP_WO(4, float, float, false, false)
        S3DSP_WO(5, float, float, false, true)
        S3DSP_WO(6, float, float, true, false)
        S3DSP_WO(7, float, float, true, true)
        S3DSP_WO(8, float, __nv_bfloat16, false, false)
        S3DSP_WO(9, float, __nv_bfloat16, false, true)
        S3DSP_WO(10, float, __nv_bfloat16, true, false)
        S3DSP_WO(11, float, __nv_bfloat16, true, true)
        S3DSP_WO(12, __nv_bfloat16, NoRes, false, false)
        S3DSP_WO(13, __nv_bfloat16, NoRes, false, true)
        S3DSP_WO(14, __nv_bfloat16, NoRes, true, false)
        S3DSP_WO(15, __nv_bfloat16, NoRes, true, true)
        S3DSP_WO(16, __nv_bfloat16, float, false, false)
        S3DSP_WO(17, __nv_bfloat16, float, false, true)
        S3DSP_WO(18, __nv_bfloat16, float, true, false)
        S3DSP_WO(19, __nv_bfloat16, float, true, true)
        S3DSP_WO(20, __nv_bfloat16, __nv_bfloat16, false, false)
        S3DSP_WO(21, __nv_bfloat16, __nv_bfloat16, false, true)
        S3DSP_WO(22, __nv_bfloat16, __nv_bfloat16, true, false)
        S3DSP_WO(23, __nv_bfloat16, __nv_bfloat16, true, true)
#undef S3DSP_WO
        default:
            writeout_generic(p, stage_out, ostride, lane_base, lane, m0, n0, limit, nrows, bias4,
                             stats ? colw : nullptr);
    }
    // deterministic GroupNorm partials of the tile from the write-out's
    // per-warp column sums
    if (stats && gn_slot) {
        bar();
        gn_tile_partials<kWarps, kWarps * 32>(colp, p.bn, n0, limit, gs, p.gn_groups, tid, gn_slot, p.gn_store != 0,
                                              bar);
    }
}

// cuTensorMapEncodeTiled through the runtime (no -lcuda)
inline PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
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


}  // namespace tc
}  // namespace s3dsp
