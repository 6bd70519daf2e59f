// BF16 implicit-gather sparse convolution with a per-tile input halo, for the
// narrow layers of the decoders (64-256 input channels, at most 128 output
// channels: the mesh decoder's upper levels, where most rows are).
//
// A 128-row tile of a submanifold conv gathers kvol x 128 neighbour rows, but
// for a locally ordered coordinate list (sorted, or children after their
// parent) those gathers hit few distinct input rows: on a 64^3 shell
// subdivided twice (970k rows) 318 on average and 380 at most per tile,
// against 3,456 gathers; a subdivide conv (in_shift = 3, parents) ~100. The
// kernel loads each distinct row once, all of its channels, into a shared-
// memory halo and builds every kernel offset's A tile from there with 16-byte
// shared loads and stores, so the L2 -> SM row traffic drops ~10x and the
// per-step row gather becomes a short, local shared-memory copy.
//
// One CTA per 128-row tile (tcgen05 cta_group::1, M = 128, N = the whole
// layer width, BN <= 128); two CTAs per SM where the halo fits in half the
// shared memory, so one CTA's prologue and epilogue overlap the other's main
// loop.
//  * prologue (warps 0-7): reads the tile's kvol x 128 map entries, finds the
//    distinct source rows with a shared-memory hash set (the first insert
//    takes the next halo slot), resolves a [kvol][128] table of halo slots,
//    and loads the halo by cp.async. A tile that references more distinct
//    rows than the halo holds (an unordered coordinate list) gathers its rows
//    from global memory instead: the same results, more traffic.
//  * main loop over (64-channel chunk, active offset) steps: warps 0-7 write
//    the step's 128 rows into the ring stage (zeros for a missing neighbour,
//    the 128-byte swizzle the MMA descriptor describes), make the writes
//    visible to the tensor core's proxy and arrive on the stage's barrier;
//    warps 8-11 load the weight tile by TMA (issued from the first stages on,
//    while the prologue runs); warp 12 issues 4 tcgen05.mma per step and
//    frees the stage with tcgen05.commit.
//  * epilogue (warps 0-7): the accumulator goes TMEM -> shared memory -> out
//    through the write-out shared with the other kernels (bias, residual,
//    SiLU / GELU, deterministic GroupNorm partial sums).
//
// Every mbarrier wait is bounded (about two seconds); on a timeout the CTA
// records kErrPipelineTimeout, skips the rest of its work, still passes every
// named barrier the other threads pass, and frees its TMEM.
//
// Reference: the GGML get_rows + mul_mat chain of the SLat conv
// (slat_flow_graph.cpp:112-155) and the mesh decoder's per-offset conv
// (mesh_decoder_graph.cpp:81-103); in_shift = 3 reads the parent row of a
// child (repeat_children, mesh_decoder_graph.cpp:32-38) without building it.
#include "s3dsp_internal.h"
#include "tc_common.cuh"

using namespace s3dsp;
using namespace s3dsp::tc;

namespace {

constexpr int kProdWarps = 8;           // halo / A-assembly / epilogue warps
constexpr int kProd = kProdWarps * 32;  // 256 threads
constexpr int kBWarp0 = 8;              // first weight-TMA warp
constexpr int kMaxBWarps = 4;
constexpr int kMmaWarp = 12;
constexpr int kThreads = 13 * 32;
constexpr int kKC = 64;                 // channels per step: 128-byte rows
constexpr int kRowB = 2 * kKC;
constexpr int kAStage = 128 * kRowB;    // 16 KB of A rows per stage
constexpr int kMaxKvol = 27;
constexpr int kMaxChunks = 4;           // input channels <= 256
constexpr int kHashSlots = 2048;        // distinct-row hash set (prologue only), >= 2x the largest halo
constexpr int kMaxHalo = 1000;
constexpr uint16_t kNoSlot = 0xFFFF;
constexpr int kEPer = (kMaxKvol * 128 + kProd - 1) / kProd;  // map entries per producer thread
constexpr int kMaxProbe = 64;  // linear-probe limit of the hash set (its load stays <= 0.5)
// per-SM shared memory of a B200 (228 KB) less the 1 KB each CTA reserves
constexpr size_t kSmemPerSm = 233472;

struct HaloParams {
    const __nv_bfloat16* in;    // [n_in, cin] bf16
    int cin;
    int in_shift;
    const int32_t* nbr;         // [kvol][n_out]
    const uint32_t* tile_mask;  // [n_tiles] or null
    int kvol;
    int kchunks;                // 64-channel chunks of the input
    int cout_pad;
    int bn;
    int nb;                     // weight TMA issuers
    int stages;
    int halo_cap;               // halo rows (all chunks of each)
    uint32_t idesc;
    const float* bias;
    const void* residual;
    uint32_t res_dtype;
    int res_shift;
    void* out;
    uint32_t out_dtype;
    int64_t n_out;
    int64_t n_tiles;
    int cout;
    uint32_t flags;
    double* gn_partials;
    int gn_store;
    int gn_groups;
    uint32_t* status;
    const void* w;              // packed weights (for the L2 prefetch before the dependency wait)
    uint64_t w_bytes;
};

__device__ __forceinline__ void prod_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ void sts128(uint32_t a, uint4 v) {
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}
__device__ __forceinline__ void mbar_arrive_local(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// 11-bit multiplicative hash of a row index
__device__ __forceinline__ uint32_t row_hash(int32_t v) { return ((uint32_t)v * 0x9E3779B1u) >> 21; }

// Shared-memory layout, in bytes from the 1024-aligned base. Region 0 holds
// the ring (A stages, then B stages) and the halo during the main loop, the
// hash set (inside the A stages) during the prologue, and the f32 output tile
// with the GroupNorm column sums in the epilogue; the slot table and the
// barriers follow it.
struct HaloLayout {
    size_t b, halo, local, bars, total;
};
__host__ __device__ inline size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
__host__ __device__ inline HaloLayout halo_layout(int stages, int bn, int halo_cap, int kchunks, int kvol) {
    HaloLayout L;
    L.b = (size_t)stages * kAStage;
    L.halo = L.b + (size_t)stages * bn * kRowB;
    const size_t main_bytes = L.halo + (size_t)halo_cap * kchunks * kRowB;
    const size_t epi = (size_t)128 * (bn + 4) * 4 + (size_t)kProdWarps * bn * 16;
    L.local = round_up(main_bytes > epi ? main_bytes : epi, 16);  // uint16 [kvol][128]
    L.bars = round_up(L.local + (size_t)kvol * 128 * 2, 16);      // full[S], empty[S], accum, words
    L.total = L.bars + (size_t)(2 * stages + 1) * 8 + 16;
    return L;
}

__global__ void __launch_bounds__(kThreads, 2) conv_halo_kernel(const HaloParams p, const __grid_constant__ CUtensorMap wmap) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int S = p.stages;
    const int H = p.halo_cap;
    const int bstage = p.bn * kRowB;
    const HaloLayout L = halo_layout(S, p.bn, H, p.kchunks, p.kvol);
    uint8_t* sA = smem;
    uint8_t* sB = smem + L.b;
    uint8_t* halo = smem + L.halo;  // chunk-major: chunk kc of halo row h at (kc * H + h) * 128
    uint16_t* local = reinterpret_cast<uint16_t*>(smem + L.local);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
    uint64_t* empty = full + S;
    uint64_t* accum = empty + S;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(accum + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
    int* halo_cnt = reinterpret_cast<int*>(tmem_holder + 2);
    // prologue scratch in the A stages (12 KB; nothing else writes them before the main loop)
    int32_t* hkeys = reinterpret_cast<int32_t*>(sA);
    uint16_t* hids = reinterpret_cast<uint16_t*>(hkeys + kHashSlots);

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int64_t tile = blockIdx.x;
    const int64_t m0 = tile * 128;
    const int n0 = blockIdx.y * p.bn;
    const uint32_t tcols = p.bn <= 32 ? 32u : p.bn <= 64 ? 64u : 128u;

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            // one arrival per producer thread (a plain arrive after its shared
            // stores, or its cp.async completions) and one expect_tx per weight issuer
            mbar_init(smem_u32(full + s), kProd + p.nb);
            mbar_init(smem_u32(empty + s), 1);
        }
        mbar_init(smem_u32(accum), 1);
        *abort_flag = 0;
        *halo_cnt = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                     "r"(tcols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // the weights do not depend on the previous kernel: start bringing this
    // CTA's share into L2 while it finishes
    if (tid == 32) prefetch_share_l2(p.w, p.w_bytes, blockIdx.y * gridDim.x + blockIdx.x, gridDim.x * gridDim.y);
    if (warp == 2) prefetch_lines_l2(p.bias, (uint64_t)p.cout * 4, lane);  // read by the epilogue
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    // everything above touched shared memory, TMEM, parameters and the L2 hint only
    pdl_wait();
    pdl_trigger();
    uint32_t mask = 0x7ffffffu;
    if (p.tile_mask) mask = tile < p.n_tiles ? p.tile_mask[tile] : 0u;
    mask &= (1u << p.kvol) - 1u;
    const int n_off = __popc(mask);
    const int T = n_off * p.kchunks;

    bool prod_ok = true;
    if (warp < kProdWarps) {
        // ============ prologue: the tile's distinct source rows ============
        for (int e = tid; e < kHashSlots; e += kProd) hkeys[e] = -1;
        prod_bar();
        const int n_e = p.kvol * 128;
        // this thread's map entries e = tid + 256 j: every load issued before any is used
        int32_t src[kEPer];
#pragma unroll
        for (int j = 0; j < kEPer; ++j) {
            const int e = tid + kProd * j;
            const int o = e >> 7, r = e & 127;
            src[j] = -1;
            if (e < n_e && ((mask >> o) & 1u) && m0 + r < p.n_out) src[j] = __ldg(p.nbr + (int64_t)o * p.n_out + m0 + r);
        }
        // pass 1a: the first probe of every entry, all in flight at once. Bit j
        // of `fresh`: entry j inserted its row; of `coll`: its slot holds another row
        uint32_t fresh = 0u, coll = 0u;
        uint16_t hpos[kEPer];
#pragma unroll
        for (int j = 0; j < kEPer; ++j) {
            src[j] = src[j] < 0 ? -1 : src[j] >> p.in_shift;
            hpos[j] = kNoSlot;
            if (src[j] >= 0) {
                const uint32_t h = row_hash(src[j]);
                const int32_t prev = atomicCAS(hkeys + h, -1, src[j]);
                hpos[j] = (uint16_t)h;
                if (prev == -1)
                    fresh |= 1u << j;
                else if (prev != src[j])
                    coll |= 1u << j;
            }
        }
        // pass 1b: linear probing for the rest. A probe longer than kMaxProbe
        // (a set filled by an unordered tile) gives the tile up to global memory
        bool give_up = false;
#pragma unroll
        for (int j = 0; j < kEPer; ++j) {
            if (!((coll >> j) & 1u)) continue;
            uint32_t h = hpos[j];
            hpos[j] = kNoSlot;
            for (int probe = 1; probe < kMaxProbe; ++probe) {
                h = (h + 1) & (kHashSlots - 1);
                const int32_t prev = atomicCAS(hkeys + h, -1, src[j]);
                if (prev == -1 || prev == src[j]) {
                    if (prev == -1) fresh |= 1u << j;
                    hpos[j] = (uint16_t)h;
                    break;
                }
            }
            give_up |= hpos[j] == kNoSlot;
        }
        // halo slots for the rows this thread inserted (one atomic per thread),
        // and their loads (every chunk) start at once
        int id = fresh ? atomicAdd(halo_cnt, __popc(fresh)) : 0;
        if (give_up) atomicAdd(halo_cnt, 1 << 20);
        const uint32_t hb0 = smem_u32(halo);
#pragma unroll
        for (int j = 0; j < kEPer; ++j) {
            if (!((fresh >> j) & 1u)) continue;
            hids[hpos[j]] = (uint16_t)min(id, (int)kNoSlot);
            if (id < H) {
                const __nv_bfloat16* row = p.in + (int64_t)src[j] * p.cin;
                for (int kc = 0; kc < p.kchunks; ++kc)
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        const int k0 = kc * kKC + c * 8;
                        const bool kin = k0 < p.cin;
                        cp_async_16(hb0 + (uint32_t)((kc * H + id) * kRowB + c * 16), kin ? row + k0 : p.in,
                                    kin ? 16u : 0u);
                    }
            }
            ++id;
        }
        prod_bar();
        const int cnt = *halo_cnt;
        const bool use_halo = cnt <= H;
        // pass 2: each entry's halo slot (kNoSlot: no neighbour)
        if (use_halo) {
#pragma unroll
            for (int j = 0; j < kEPer; ++j) {
                const int e = tid + kProd * j;
                if (e < n_e) local[e] = hpos[j] == kNoSlot ? kNoSlot : hids[hpos[j]];
            }
        }
        const int c16 = tid & 7;  // 16-byte chunk of a row
        const int rg = tid >> 3;  // rows rg + 32 i
        asm volatile("cp.async.wait_all;" ::: "memory");
        prod_bar();  // slots resolved, the halo landed; the hash set is dead

        // ============ main loop: one A tile per (chunk, active offset) step ============
        const uint32_t a_ring = smem_u32(sA);
        const uint32_t hb = smem_u32(halo) + (uint32_t)c16 * 16u;
        int it = 0;
        for (int kc = 0; kc < p.kchunks && prod_ok; ++kc) {
            const uint32_t hbk = hb + (uint32_t)(kc * H) * kRowB;
            const int k0 = kc * kKC + c16 * 8;
            uint32_t mrem = mask;
            for (int q = 0; q < n_off; ++q, ++it) {
                const int o = __ffs(mrem) - 1;
                mrem &= mrem - 1;
                const int s = it % S;
                const uint32_t ph = (uint32_t)(it / S) & 1u;
                if (!mbar_wait(smem_u32(empty + s), ph ^ 1u, abort_flag, p.status)) {
                    prod_ok = false;
                    break;
                }
                const uint32_t a_base = a_ring + (uint32_t)(s * kAStage);
                if (use_halo) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int row = rg + 32 * i;
                        const uint16_t slot = local[o * 128 + row];
                        uint4 v = make_uint4(0u, 0u, 0u, 0u);
                        if (slot != kNoSlot) v = lds128(hbk + (uint32_t)slot * kRowB);
                        sts128(a_base + (uint32_t)(row * kRowB + ((c16 ^ kmajor_swz<kKC>(row)) << 4)), v);
                    }
                    // generic-proxy writes, read by the tensor core (async proxy)
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    mbar_arrive_local(smem_u32(full + s));
                } else {
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int row = rg + 32 * i;
                        const int64_t r = m0 + row;
                        int32_t src = -1;
                        if (r < p.n_out) src = __ldg(p.nbr + (int64_t)o * p.n_out + r);
                        const bool valid = src >= 0 && k0 < p.cin;
                        const void* g = valid ? (const void*)(p.in + (int64_t)(src >> p.in_shift) * p.cin + k0)
                                              : (const void*)p.in;
                        cp_async_16(a_base + (uint32_t)(row * kRowB + ((c16 ^ kmajor_swz<kKC>(row)) << 4)), g,
                                    valid ? 16u : 0u);
                    }
                    cp_async_arrive_noinc(smem_u32(full + s));
                }
            }
        }
        if (p.residual && tile < p.n_tiles) {
            // the epilogue reads this tile's residual rows: start bringing them
            // into L2 now, while the last stages are still in flight
            const int esz = p.res_dtype == S3DSP_F32 ? 4 : 2;
            const int64_t r = m0 + (tid >> 1);
            const int len = min(p.bn, p.cout - n0) * esz;
            if (r < p.n_out) {
                const char* row = static_cast<const char*>(p.residual) +
                                  (((r >> p.res_shift) * p.cout + n0) * (int64_t)esz);
                for (int b = (tid & 1) * 128; b < len; b += 2 * 128)
                    asm volatile("prefetch.global.L2 [%0];" ::"l"(row + b));
            }
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
    } else if (warp < kBWarp0 + kMaxBWarps) {
        // ============ weight TMA issuers ============
        const int j = warp - kBWarp0;
        if (lane == 0 && j < p.nb) {
            const int rows = p.bn / p.nb;
            const uint32_t bytes = (uint32_t)rows * kRowB;
            int it = 0;
            bool ok = true;
            for (int kc = 0; kc < p.kchunks && ok; ++kc) {
                uint32_t mrem = mask;
                for (int q = 0; q < n_off; ++q, ++it) {
                    const int o = __ffs(mrem) - 1;
                    mrem &= mrem - 1;
                    const int s = it % S;
                    const uint32_t ph = (uint32_t)(it / S) & 1u;
                    if (!mbar_wait(smem_u32(empty + s), ph ^ 1u, abort_flag, p.status)) {
                        ok = false;
                        break;
                    }
                    const uint32_t fb = smem_u32(full + s);
                    mbar_arrive_tx(fb, bytes);
                    tma_load_2d(smem_u32(sB + (size_t)s * bstage + (size_t)j * rows * kRowB), &wmap, kc * kKC,
                                o * p.cout_pad + n0 + j * rows, fb);
                }
            }
        }
        __syncwarp();
    } else if (warp == kMmaWarp) {
        // ============ MMA issuer ============
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
                for (int k = 0; k < kKC / 16; ++k)
                    mma_bf16(tmem, kmajor_desc<kKC>(a0 + 32 * k), kmajor_desc<kKC>(b0 + 32 * k), p.idesc,
                             (it > 0 || k > 0) ? 1u : 0u);
                mma_commit(smem_u32(empty + s));
            }
            if (ok && T > 0) mma_commit(smem_u32(accum));
        }
        __syncwarp();
    }

    if (warp < kProdWarps) {
        // ============ epilogue (warps 0-7) ============
        bool have_acc = T > 0 && prod_ok && mbar_wait(smem_u32(accum), 0, abort_flag, p.status);
        have_acc = __all_sync(0xffffffffu, have_acc);
        tc_fence_after();
        const int ostride = p.bn + 4;
        float* stage_out = reinterpret_cast<float*>(smem);  // reuses the ring and the halo
        // every producer is past its last halo read before the tile overwrites it
        prod_bar();
        {
            // warp w: TMEM lanes 32 * (w % 4) .. (its rows), 16-column chunks w / 4, w / 4 + 2, ...
            const int lq = warp & 3;
            float* dst = stage_out + (size_t)(32 * lq + lane) * ostride;
            const uint32_t taddr = tmem + ((uint32_t)(32 * lq) << 16);
            for (int c0 = 16 * (warp >> 2); c0 < p.bn; c0 += 16 * (kProdWarps / 4)) {
                float f[16];
                if (have_acc) {
                    tmem_ld16(taddr + (uint32_t)c0, f);
                } else {
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) f[jj] = 0.f;
                }
#pragma unroll
                for (int qq = 0; qq < 4; ++qq)
                    *reinterpret_cast<float4*>(dst + c0 + 4 * qq) =
                        make_float4(f[4 * qq], f[4 * qq + 1], f[4 * qq + 2], f[4 * qq + 3]);
            }
        }
        prod_bar();
        tile_writeout<kProdWarps>(p, smem, ostride, warp, lane, tid, m0, n0,
                                  p.gn_partials && tile < p.n_tiles ? p.gn_partials + tile * p.gn_groups * 2 : nullptr,
                                  prod_bar);
        tc_fence_before();
    }

    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tcols) : "memory");
    }
}

}  // namespace

namespace s3dsp {

// The halo kernel's plan for a layer: ring stages, halo rows and CTAs per SM.
// False when the kernel does not take the layer (no kernel map, kvol > 27,
// more than 256 input or 128 output channels). Two CTAs per SM when a halo of
// `need` rows fits in half of the SM's shared memory with a 2-stage ring, else
// one CTA with the deepest ring (4..2 stages) that still leaves 1.25 x `need`
// rows. `need` is what a 128-row tile of a locally ordered list references:
// ~400 rows at one level (a twice-subdivided 64^3 shell: 380 at most at
// C = 64, 498 at C = 128), ~140 parents for a subdivide conv (in_shift 3).
bool conv_halo_plan(int cin, int cout, int kvol, int in_shift, int* stages, int* halo_cap, int* per_sm) {
    const int cout_pad = (cout + 15) / 16 * 16;
    const int bn = tc_pick_bn(cout);
    const int kchunks = (cin + 63) / 64;
    if (kvol < 1 || kvol > kMaxKvol || cin < 1 || kchunks > kMaxChunks || bn != cout_pad || bn > 128) return false;
    const int need = in_shift >= 3 ? 160 : 400;
    auto fit = [&](int s, size_t limit) {
        int lo = 0, hi = kMaxHalo;
        while (lo < hi) {  // the largest halo that fits
            const int mid = (lo + hi + 1) / 2;
            if (1024 + halo_layout(s, bn, mid, kchunks, kvol).total <= limit)
                lo = mid;
            else
                hi = mid - 1;
        }
        return lo;
    };
    int h = fit(2, kSmemPerSm / 2 - 1024);
    if (h >= need) {
        *stages = 2;
        *halo_cap = h;
        *per_sm = 2;
        return true;
    }
    for (int s = 4; s >= 2; --s) {
        h = fit(s, (size_t)kSmemOptIn);
        if (h >= need + need / 4 || s == 2) {
            *stages = s;
            *halo_cap = h;
            *per_sm = 1;
            return h > 0;
        }
    }
    return false;
}

cudaError_t launch_conv_halo(s3dsp_context* ctx, const s3dsp_kmap* kmap, int kvol, const __nv_bfloat16* in, int cin,
                             int in_shift, const __nv_bfloat16* w, const float* bias, const void* residual,
                             uint32_t res_dtype, int res_shift, void* out, uint32_t out_dtype, int64_t n_out, int cout,
                             uint32_t flags, double* gn_partials, int gn_groups, char* error, uint64_t error_capacity,
                             s3d_status* st) {
    *st = S3D_OK;
    int stages = 0, cap = 0, per_sm = 0;
    if (!kmap || !conv_halo_plan(cin, cout, kvol, in_shift, &stages, &cap, &per_sm)) {
        *st = fail(error, error_capacity, S3D_INVALID_ARGUMENT,
                   "halo conv: needs a kernel map (kvol <= 27), cin <= 256 and cout <= 128");
        return cudaErrorInvalidValue;
    }
    const int cout_pad = (cout + 15) / 16 * 16;
    const int cin_pad = (cin + 63) / 64 * 64;
    const int bn = cout_pad;
    const int nb = (bn % 32 == 0) ? 4 : (bn % 16 == 0) ? 2 : 1;
    const int64_t tiles = (n_out + 127) / 128;

    auto encode = get_encode_fn();
    if (!encode) {
        *st = fail(error, error_capacity, S3D_INTERNAL_ERROR, "cuTensorMapEncodeTiled unavailable");
        return cudaErrorNotSupported;
    }
    CUtensorMap wmap;
    {
        const cuuint64_t dims[2] = {(cuuint64_t)cin_pad, (cuuint64_t)kvol * (cuuint64_t)cout_pad};
        const cuuint64_t strides[1] = {(cuuint64_t)cin_pad * 2};
        const cuuint32_t box[2] = {(cuuint32_t)kKC, (cuuint32_t)(bn / nb)};
        const cuuint32_t estr[2] = {1, 1};
        CUresult cr = encode(&wmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<__nv_bfloat16*>(w), dims, strides,
                             box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (cr != CUDA_SUCCESS) {
            *st = fail(error, error_capacity, S3D_INTERNAL_ERROR, "weight tensor map failed (%d)", (int)cr);
            return cudaErrorInvalidValue;
        }
    }
    HaloParams p;
    p.in = in;
    p.cin = cin;
    p.in_shift = in_shift;
    p.nbr = kmap->nbr;
    p.tile_mask = kmap->tile_mask;
    p.kvol = kvol;
    p.kchunks = cin_pad / kKC;
    p.cout_pad = cout_pad;
    p.bn = bn;
    p.nb = nb;
    p.stages = stages;
    p.halo_cap = cap;
    // f32 accumulator, A = B = BF16, both K-major, N = bn, M = 128
    p.idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(bn >> 3) << 17) | ((128u >> 4) << 24);
    p.bias = bias;
    p.residual = residual;
    p.res_dtype = res_dtype;
    p.res_shift = res_shift;
    p.out = out;
    p.out_dtype = out_dtype;
    p.n_out = n_out;
    p.n_tiles = tiles;
    p.cout = cout;
    p.flags = flags;
    p.gn_partials = gn_partials;
    p.gn_store = 1;  // one column tile covers every channel
    p.gn_groups = gn_groups;
    p.status = ctx->d_status;
    p.w = w;
    p.w_bytes = (uint64_t)kvol * (uint64_t)cout_pad * (uint64_t)cin_pad * 2;

    const size_t smem = 1024 + halo_layout(stages, bn, cap, p.kchunks, kvol).total;
    static std::atomic<uint64_t> optin{0};
    cudaError_t e = smem_optin((const void*)conv_halo_kernel, ctx->device, optin);
    if (e == cudaSuccess && smem > (size_t)kSmemOptIn) e = cudaErrorInvalidValue;
    if (e != cudaSuccess) return e;
    e = launch_pdl(conv_halo_kernel, dim3((unsigned)tiles, 1u), dim3(kThreads), smem, ctx->stream, p, wmap);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace s3dsp
