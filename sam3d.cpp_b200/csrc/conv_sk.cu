// BF16 implicit-gather sparse convolution, stream-K form: the default
// tensor-core path.
//
// Work tile: 256 output rows x BN output channels, held as two 128-row f32
// accumulators in TMEM (columns [0, BN) and [H, H + BN), H = the allocation
// half). Each weight tile that TMA brings in feeds both accumulators, so a
// reduction step moves 32 KB of gathered rows + BN x 128 B of weights for
// 2 x 128 x BN x 64 MACs. The per-SM copy rate, not L2 bandwidth, bounds
// this kernel (L2 runs at about a fifth of its peak), so bytes per MAC per
// SM is what the tile shape minimises.
//
// Stream-K: the iteration space (work tile, kernel offset) of U = tiles x
// kvol units is cut into `grid` (= number of SMs, fewer for small problems)
// contiguous ranges of equal length, one per CTA, so every SM gets the same
// number of reduction steps whatever the tile count. A CTA walks its range
// as segments (one work tile each). A tile covered by one CTA runs the
// epilogue straight from TMEM. A tile split over k CTAs ("pieces") is fixed
// up without any waiting: each piece stores its raw accumulator to a
// workspace slot, then bumps the tile's counter; the piece that arrives
// last sums the k slots in piece order (so the result does not depend on
// which CTA finished last) and runs the epilogue. Nothing spins on another
// CTA, so no co-residency is assumed.
//
// Warp roles (672 threads) as in the 128-row kernel: warps 0-15 gather A by
// cp.async (4 rows x 16 B per thread per step; each thread reads the map
// entries of its own rows from global memory one kernel offset ahead, so a
// segment starts gathering at once) and then run the epilogue
// (warp w: TMEM lanes 32*(w%4).., column chunks w/4, w/4+4, ...; write-out
// rows 8w..8w+7), warps 16-19 issue the weight TMA loads, warp 20 owns TMEM
// and issues 8 tcgen05.mma (M=128, N=BN, K=16) per step. Waits are bounded
// (2 s of %globaltimer); a timeout sets kErrPipelineTimeout and the CTA
// leaves through the common teardown.
//
// Replaces the same reference code as the 128-row kernel: the GGML
// get_rows + mul_mat chains of slat_flow_graph.cpp:112-155 and
// mesh_decoder_graph.cpp:81-103 (in_shift = 3 is repeat_children,
// mesh_decoder_graph.cpp:32-38, without materialising it).
#include "s3dsp_internal.h"
#include "tc_common.cuh"

using namespace s3dsp;
using namespace s3dsp::tc;

namespace {

constexpr int kProdWarps = 16;        // A gather + epilogue warps (512 threads)
constexpr int kEpiThreads = kProdWarps * 32;
constexpr int kBWarp0 = 16;           // first weight-TMA warp
constexpr int kMaxBWarps = 4;
constexpr int kMmaWarp = 20;
constexpr int kThreads = 21 * 32;
constexpr int kKC = 64;  // channels per pipeline stage (128-byte rows, SWIZZLE_128B; 32 measured slower)
constexpr int kAHalf = 128 * 2 * kKC;  // the second accumulator's rows start here in an A stage
constexpr int kSmemMax = kSmemOptIn;

struct SkParams {
    const __nv_bfloat16* in;
    const __nv_bfloat16* in_b;  // second source (channels [cin_a, cin)) or null
    int cin_a;
    int cin;
    int in_shift;
    const int32_t* nbr;         // [kvol][n_out] or null (identity)
    const uint32_t* tile_mask;  // [128-row tiles] or null
    int kvol;
    int kchunks;                // kKC-channel reduction chunks per offset
    int cout_pad;               // packed weight rows per offset
    int bn;
    int nb;                     // weight TMA loads per stage
    int stages;
    uint32_t tcols;             // TMEM columns allocated
    uint32_t thalf;             // column of the second accumulator
    uint32_t idesc;
    const float* bias;
    const void* residual;
    uint32_t res_dtype;
    int res_shift;
    void* out;
    uint32_t out_dtype;
    int64_t n_out;
    int64_t n_tiles;            // 128-row tiles (GroupNorm partial slots)
    int nnb;                    // column blocks per 256-row tile
    int64_t units;              // work tiles x kvol
    int grid;
    int csplit;                 // 2: split-K over CTA pairs (clusters of 2, kRows = 256); 1: stream-K
    int gn_store;               // one column block: GroupNorm partials stored, not added onto zeroed slots
    float* ws;                  // [2 * grid][rows / 128][bn / 16][4][128] float4 raw accumulators, or null
    uint32_t* counters;         // [work tiles] pieces arrived, zeroed before launch
    int cout;
    uint32_t flags;
    double* gn_partials;
    int gn_groups;
    uint32_t* status;
    const void* w;              // packed weights (for the L2 prefetch before the dependency wait)
    uint64_t w_bytes;
};

__device__ __forceinline__ int64_t unit_begin(const SkParams& p, int i) {
    return (int64_t)i * p.units / p.grid;
}
// the CTA whose unit range holds unit u
__device__ __forceinline__ int cta_of(const SkParams& p, int64_t u) {
    int i = (int)(u * p.grid / p.units);
    while (i + 1 < p.grid && unit_begin(p, i + 1) <= u) ++i;
    while (i > 0 && unit_begin(p, i) > u) --i;
    return i;
}
// workspace slot of CTA i's piece of work tile wt: a CTA is split-owner of at
// most its first and its last tile
__device__ __forceinline__ int64_t ws_slot(const SkParams& p, int i, int64_t wt) {
    return 2 * (int64_t)i + ((unit_begin(p, i) / p.kvol) == wt ? 0 : 1);
}
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 512;" ::: "memory"); }

// the area after the staged f32 tile: per-warp GroupNorm column sums (f64 pairs),
// or, for split-K pairs, the staging area of the larger half of the columns
// (128 rows of 4 float4s per 16-column chunk, plus one float4 of padding)
__host__ __device__ constexpr size_t colsum_bytes(int bn) {
    const size_t sums = (size_t)kProdWarps * bn * 16;
    const size_t stage = (size_t)128 * (4 * ((bn / 16 + 1) / 2) + 1) * 16;
    return sums > stage ? sums : stage;
}



// kRows = 256: two 128-row accumulators per work tile; 128: one. kTwo: the
// input is the channel concat of two sources (a separate instance, so the
// one-source gather keeps its shorter address path).
template <int kRows, bool kTwo = false>
__global__ void __launch_bounds__(kThreads, 1) conv_sk_kernel(const SkParams p, const __grid_constant__ CUtensorMap wmap) {
    constexpr int kSub = kRows / 128;              // 128-row accumulators per work tile
    constexpr int kAStage = kRows * 2 * kKC;       // bytes: kRows gathered rows x kKC bf16
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int S = p.stages;
    const int bstage = p.bn * 2 * kKC;
    const int ostride = p.bn + 4;  // staged f32 row stride (floats)
    // layout: region0 = max(ring A | ring B, epilogue tile | GN column sums),
    // then barriers, tmem holder, flags
    const size_t ring = (size_t)S * (kAStage + bstage);
    const size_t epi = (size_t)128 * ostride * 4 + colsum_bytes(p.bn);
    uint8_t* sA = smem;
    uint8_t* sB = smem + (size_t)S * kAStage;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (ring > epi ? ring : epi));
    uint64_t* empty = full + S;
    uint64_t* accum = empty + S;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(accum + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
    volatile int* owner_flag = abort_flag + 1;
    float* stage_out = reinterpret_cast<float*>(smem);
    double* colp = reinterpret_cast<double*>(smem + (size_t)128 * ostride * 4);  // [16][bn][2]

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int me = blockIdx.x;

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(smem_u32(full + s), kEpiThreads + p.nb);
            mbar_init(smem_u32(empty + s), 1);
        }
        mbar_init(smem_u32(accum), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                     "r"(p.tcols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // the weights do not depend on the previous kernel: start bringing this
    // CTA's share into L2 while it finishes
    if (tid == 32) prefetch_share_l2(p.w, p.w_bytes, (uint32_t)me, (uint32_t)p.grid);
    if (warp == 2) prefetch_lines_l2(p.bias, (uint64_t)p.cout * 4, lane);  // read by the epilogue
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    // everything above touched shared memory, TMEM, parameters and the L2 hint only
    pdl_wait();
    pdl_trigger();

    uint32_t it = 0;      // pipeline step counter, identical in every role
    uint32_t acc_ph = 0;  // accum barrier phase
    // split-K pairs: the CTA pair (a cluster of 2) shares work tile me / 2, one
    // segment each; rank r keeps its half of the tile's kernel offsets and
    // finishes accumulator r (rows 128 r ..) with the peer's part added in
    const bool csp = kRows == 256 && p.csplit == 2;
    const uint32_t crank = csp ? cluster_rank() : 0u;
    const int64_t u_end = csp ? 1 : unit_begin(p, me + 1);
    for (int64_t u = csp ? 0 : unit_begin(p, me); u < u_end;) {
        const int64_t wt = csp ? (int64_t)(me >> 1) : u / p.kvol;
        const int64_t seg_end = csp ? 1 : min(u_end, (wt + 1) * p.kvol);
        const int ob = csp ? 0 : (int)(u - wt * p.kvol), oe = csp ? p.kvol : (int)(seg_end - wt * p.kvol);
        u = seg_end;
        const int64_t st = wt / p.nnb;
        const int n0 = (int)(wt - st * p.nnb) * p.bn;
        const int64_t m0 = st * kRows;

        uint32_t mask = 1u;
        if (p.nbr) {
            mask = 0xffffffffu;
            if (p.tile_mask) {
                mask = 0u;
#pragma unroll
                for (int j = 0; j < kSub; ++j)
                    if (kSub * st + j < p.n_tiles) mask |= p.tile_mask[kSub * st + j];
            }
        }
        mask &= (oe >= 32 ? 0xffffffffu : ((1u << oe) - 1u)) & ~((1u << ob) - 1u);
        // this CTA's reduction steps: T steps of kKC channels, starting at
        // chunk kc0 of the first offset left in `mask`
        int T = __popc(mask) * p.kchunks;
        int kc0 = 0;
        if (csp) {
            // rank 0: the first ceil(steps / 2) steps of the tile's offsets,
            // rank 1: the rest (it may start inside an offset)
            const int half = (T + 1) / 2;
            if (crank) {
                for (int q = half / p.kchunks; q > 0; --q) mask &= mask - 1u;
                kc0 = half % p.kchunks;
                T -= half;
            } else {
                T = half;
            }
        }

        bool prod_ok = true;
        if (warp < kProdWarps) {
            // ============ A producers: cp.async gathers ============
            constexpr int kCpr = kKC / 8;         // 16-byte chunks per row
            constexpr int kRowStep = 512 / kCpr;  // rows covered by one pass of the 512 threads
            constexpr int kMine = kRows / kRowStep;  // rows of this thread: rg + kRowStep * i
            const int c16 = tid & (kCpr - 1);
            const int rg = tid / kCpr;
            // the map entries of this thread's rows for kernel offset o (source row, or -1)
            auto load_idx = [&](int o, int32_t (&dst)[kMine]) {
#pragma unroll
                for (int i = 0; i < kMine; ++i) {
                    const int64_t r = m0 + rg + kRowStep * i;
                    int32_t src = -1;
                    if (r < p.n_out) src = p.nbr ? __ldg(p.nbr + (int64_t)o * p.n_out + r) : (int32_t)r;
                    dst[i] = src < 0 ? -1 : (src >> p.in_shift);
                }
            };
            uint32_t mrem = mask;
            int32_t cur[kMine], nxt[kMine];
            if (mrem) {
                load_idx(__ffs(mrem) - 1, nxt);
                mrem &= mrem - 1;
            }
            for (int j = 0; j < T; ++j) {
                const uint32_t pit = it + (uint32_t)j;
                const int s = (int)(pit % (uint32_t)S);
                const uint32_t ph = (pit / (uint32_t)S) & 1u;
                const int kc = (kc0 + j) % p.kchunks;
                if (kc == 0 || j == 0) {  // next kernel offset: its entries were loaded one offset ago
#pragma unroll
                    for (int i = 0; i < kMine; ++i) cur[i] = nxt[i];
                    if (mrem) {
                        load_idx(__ffs(mrem) - 1, nxt);
                        mrem &= mrem - 1;
                    }
                }
                if (!mbar_wait(smem_u32(empty + s), ph ^ 1u, abort_flag, p.status)) {
                    prod_ok = false;
                    break;
                }
                const int k0 = kc * kKC + c16 * 8;
                const uint32_t a_base = smem_u32(sA + (size_t)s * kAStage);
                // channel concat of two sources: the source holding channel k0
                // and its row stride, fixed for the whole stage
                const bool from_a = !kTwo || k0 < p.cin_a;
                const __nv_bfloat16* base = from_a ? p.in + k0 : p.in_b + (k0 - p.cin_a);
                const int64_t ld = kTwo ? (from_a ? p.cin_a : p.cin - p.cin_a) : p.cin;
#pragma unroll
                for (int i = 0; i < kMine; ++i) {
                    const int row = rg + kRowStep * i;
                    const int32_t src = cur[i];
                    const bool valid = src >= 0 && k0 < p.cin;
                    const void* g = valid ? (const void*)(base + (int64_t)src * ld) : (const void*)p.in;
                    cp_async_16(a_base + row * (2 * kKC) + ((c16 ^ kmajor_swz<kKC>(row)) << 4), g, valid ? 16u : 0u);
                }
                cp_async_arrive_noinc(smem_u32(full + s));
            }
        } else if (warp < kBWarp0 + kMaxBWarps) {
            // ============ weight TMA issuers ============
            const int jw = warp - kBWarp0;
            if (lane == 0 && jw < p.nb) {
                const int rows = p.bn / p.nb;
                const uint32_t bytes = (uint32_t)rows * 2 * kKC;
                uint32_t mrem = mask;
                int o = 0;
                for (int j = 0; j < T; ++j) {
                    const uint32_t pit = it + (uint32_t)j;
                    const int s = (int)(pit % (uint32_t)S);
                    const uint32_t ph = (pit / (uint32_t)S) & 1u;
                    const int kc = (kc0 + j) % p.kchunks;
                    if (kc == 0 || j == 0) {
                        o = __ffs(mrem) - 1;
                        mrem &= mrem - 1;
                    }
                    if (!mbar_wait(smem_u32(empty + s), ph ^ 1u, abort_flag, p.status)) break;
                    const uint32_t fb = smem_u32(full + s);
                    mbar_arrive_tx(fb, bytes);
                    tma_load_2d(smem_u32(sB + (size_t)s * bstage + (size_t)jw * rows * 2 * kKC), &wmap, kc * kKC,
                                o * p.cout_pad + n0 + jw * rows, fb);
                }
            }
            __syncwarp();
        } else if (warp == kMmaWarp) {
            // ============ MMA issuer: two M=128 accumulators per weight tile ============
            if (lane == 0) {
                bool ok = true;
                for (int j = 0; j < T; ++j) {
                    const uint32_t pit = it + (uint32_t)j;
                    const int s = (int)(pit % (uint32_t)S);
                    const uint32_t ph = (pit / (uint32_t)S) & 1u;
                    if (!mbar_wait(smem_u32(full + s), ph, abort_flag, p.status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + (size_t)s * kAStage);
                    const uint32_t b0 = smem_u32(sB + (size_t)s * bstage);
#pragma unroll
                    for (int k = 0; k < kKC / 16; ++k) {
                        const uint32_t acc = (j > 0 || k > 0) ? 1u : 0u;
                        const uint64_t bd = kmajor_desc<kKC>(b0 + 32 * k);
                        mma_bf16(tmem, kmajor_desc<kKC>(a0 + 32 * k), bd, p.idesc, acc);
                        if constexpr (kSub == 2)
                            mma_bf16(tmem + p.thalf, kmajor_desc<kKC>(a0 + kAHalf + 32 * k), bd, p.idesc, acc);
                    }
                    mma_commit(smem_u32(empty + s));
                }
                if (ok && T > 0) mma_commit(smem_u32(accum));
            }
            __syncwarp();
        }
        it += (uint32_t)T;

        if (warp < kProdWarps && p.residual) {
            // the epilogue reads this work tile's residual rows: start bringing
            // them into L2 while the last MMAs finish
            const int esz = p.res_dtype == S3DSP_F32 ? 4 : 2;
            constexpr int kTpr = kEpiThreads / kRows;  // threads per row
            // split-K pairs: only the rows this CTA finishes, two threads each
            const int64_t r = csp ? m0 + 128 * (int64_t)crank + (tid >> 2) : m0 + tid / kTpr;
            const int len = min(p.bn, p.cout - n0) * esz;
            if (r < p.n_out) {
                const char* row = static_cast<const char*>(p.residual) +
                                  (((r >> p.res_shift) * p.cout + n0) * (int64_t)esz);
                const int tpr = csp ? 4 : kTpr;
                for (int b = (tid % tpr) * 128; b < len; b += tpr * 128)
                    asm volatile("prefetch.global.L2 [%0];" ::"l"(row + b));
            }
        }

        // ============ epilogue (warps 0-15) ============
        const int lq = warp & 3;                  // TMEM lane quarter (rows 32*lq ..)
        const int row = 32 * lq + lane;           // accumulator row of this thread
        const uint32_t tl = tmem + ((uint32_t)(32 * lq) << 16);
        const int nch = p.bn / 16;                // 16-column chunks
        bool have_acc = false;
        if (warp < kProdWarps && T > 0) {
            have_acc = prod_ok && mbar_wait(smem_u32(accum), acc_ph, abort_flag, p.status);
            have_acc = __all_sync(0xffffffffu, have_acc);
        }
        if (csp) {
            // split-K pairs, every thread of both CTAs at the cluster barriers.
            // Once both rings are drained (the MMAs that read them completed
            // before `accum`), accumulator `crank ^ 1` goes into the peer's
            // staged f32 tile, in two halves of the columns: TMEM -> a local
            // staging area (the GroupNorm column-sum area, rows padded by 16
            // bytes) -> 16-byte distributed-shared-memory stores, a warp writing
            // 512 contiguous bytes of one row (row-scattered remote stores ran at
            // a third of the speed; remote f32 atomic adds at ~1/10). Then each
            // CTA adds its own accumulator `crank` to what it received: one add
            // per element, own + peer, so the result is the same on every run.
            float4* stg = reinterpret_cast<float4*>(colp);
            const uint32_t peer = map_to_rank(smem_u32(stage_out), crank ^ 1u);
            const int hch = nch / 2;      // chunks in the first half (the second takes the odd one)
            const int sw = 4 * (nch - hch) + 1;  // staging row stride in float4s
            cluster_sync();
            for (int h = 0; h < 2; ++h) {
                const int c_lo = h * hch, c_hi = h ? nch : hch;
                if (warp < kProdWarps) {
                    tc_fence_after();
                    for (int c = c_lo + (warp >> 2); c < c_hi; c += 4) {
                        float f[16];
#pragma unroll
                        for (int q = 0; q < 16; ++q) f[q] = 0.f;
                        if (have_acc) tmem_ld16(tl + (crank ^ 1u) * p.thalf + 16 * c, f);
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            stg[row * sw + (c - c_lo) * 4 + q] = make_float4(f[4 * q], f[4 * q + 1], f[4 * q + 2], f[4 * q + 3]);
                    }
                    epi_bar();
                    const int w4 = 4 * (c_hi - c_lo);  // float4s per row in this half
                    for (int rr = 0; rr < 8; ++rr) {
                        const int r = 8 * warp + rr;
                        for (int j = lane; j < w4; j += 32) {
                            const float4 v = stg[r * sw + j];
                            st_cluster_v4(peer + (uint32_t)(r * ostride + 16 * c_lo + 4 * j) * 4u, v.x, v.y, v.z, v.w);
                        }
                    }
                    epi_bar();  // the staging area is refilled by the next half
                }
            }
            cluster_sync();
            if (warp < kProdWarps) {
                tc_fence_after();
                for (int c = warp >> 2; c < nch; c += 4) {
                    float f[16];
#pragma unroll
                    for (int q = 0; q < 16; ++q) f[q] = 0.f;
                    if (have_acc) tmem_ld16(tl + crank * p.thalf + 16 * c, f);
                    float4* dst = reinterpret_cast<float4*>(stage_out + (size_t)row * ostride + 16 * c);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        float4 a = dst[q];
                        a.x += f[4 * q], a.y += f[4 * q + 1], a.z += f[4 * q + 2], a.w += f[4 * q + 3];
                        dst[q] = a;
                    }
                }
            }
            // the write-out's barrier after phase 1 orders these adds before it reads the tile
        }
        if (warp < kProdWarps) {
            tc_fence_after();
            const int64_t tb = wt * p.kvol;
            const int i_first = csp ? me : cta_of(p, tb), i_last = csp ? me : cta_of(p, tb + p.kvol - 1);
            const int k = i_last - i_first + 1;
            // piece pc > 0 starts inside this tile (its first tile: slot 2i); piece 0
            // may have started in an earlier tile (then this is its last: slot 2i+1)
            const int64_t slot0 = ws_slot(p, i_first, wt);
            const int64_t slot_stride = (int64_t)kRows * p.bn;
            bool owner = true;
            if (k > 1) {
                // store the raw accumulator as float4s [sub][16-column chunk][quad][row]:
                // each warp access is 512 contiguous bytes
                float* slot = p.ws + (me == i_first ? slot0 : 2 * (int64_t)me) * slot_stride;
                for (int sub = 0; sub < kSub; ++sub)
                    for (int c = warp >> 2; c < nch; c += 4) {
                        float f[16];
                        if (have_acc) {
                            tmem_ld16(tl + sub * p.thalf + 16 * c, f);
                        } else {
#pragma unroll
                            for (int q = 0; q < 16; ++q) f[q] = 0.f;
                        }
                        float4* d = reinterpret_cast<float4*>(slot) + (size_t)(sub * nch + c) * 512 + row;
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            d[q * 128] = make_float4(f[4 * q], f[4 * q + 1], f[4 * q + 2], f[4 * q + 3]);
                    }
                __threadfence();
                epi_bar();
                if (tid == 0) *owner_flag = atomicAdd(p.counters + wt, 1u) == (uint32_t)(k - 1);
                epi_bar();
                owner = *owner_flag != 0;
                if (owner) __threadfence();
            }
            if (owner) {
                const bool stats = p.gn_partials != nullptr;
                const int gs = stats ? p.cout / p.gn_groups : 1;
                const int limit = min(p.bn, p.cout - n0);
                float4 bias4[2];
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    const int col = n0 + 128 * q + 4 * lane;
                    bias4[q] = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (p.bias && 128 * q + 4 * lane < limit) {
                        bias4[q].x = __ldg(p.bias + col + 0);
                        bias4[q].y = col + 1 < p.cout ? __ldg(p.bias + col + 1) : 0.f;
                        bias4[q].z = col + 2 < p.cout ? __ldg(p.bias + col + 2) : 0.f;
                        bias4[q].w = col + 3 < p.cout ? __ldg(p.bias + col + 3) : 0.f;
                    }
                }
                const int out_k = (p.cout & 3) ? -1 : p.out_dtype == S3DSP_F32 ? 0 : p.out_dtype == S3DSP_BF16 ? 1 : -1;
                const int res_k = !p.residual ? 0 : p.res_dtype == S3DSP_F32 ? 1 : p.res_dtype == S3DSP_BF16 ? 2 : -1;
                const int silu_k = (p.flags & S3DSP_EPI_SILU) ? 1 : 0;
                const int sel = (out_k < 0 || res_k < 0 || (p.flags & S3DSP_EPI_GELU)) ? -1 : ((out_k * 3 + res_k) * 2 + silu_k) * 2 + (stats ? 1 : 0);
                const uint32_t so_base = smem_u32(stage_out);
                for (int sub = csp ? (int)crank : 0; sub < (csp ? (int)crank + 1 : kSub); ++sub) {
                    const int64_t ms = m0 + 128 * sub;
                    if (ms >= p.n_out) break;
                    // phase 1: accumulator (TMEM, or the pieces summed in piece order) -> smem tile
                    // (split-K pairs: staged already)
                    for (int c = warp >> 2; c < (csp ? 0 : nch); c += 4) {
                        float f[16];
#pragma unroll
                        for (int q = 0; q < 16; ++q) f[q] = 0.f;
                        if (k == 1) {
                            if (have_acc) tmem_ld16(tl + sub * p.thalf + 16 * c, f);
                        } else {
                            // pieces in piece order; this CTA's own piece comes from TMEM (the
                            // workspace holds the same f32 values)
                            for (int pc = 0; pc < k; ++pc) {
                                if (i_first + pc == me) {
                                    float g[16];
                                    if (have_acc) {
                                        tmem_ld16(tl + sub * p.thalf + 16 * c, g);
#pragma unroll
                                        for (int q = 0; q < 16; ++q) f[q] += g[q];
                                    }
                                    continue;
                                }
                                const int64_t sl = pc == 0 ? slot0 : 2 * (int64_t)(i_first + pc);
                                const float4* s4 = reinterpret_cast<const float4*>(p.ws + sl * slot_stride) +
                                                   (size_t)(sub * nch + c) * 512 + row;
#pragma unroll
                                for (int q = 0; q < 4; ++q) {
                                    const float4 v = __ldcg(s4 + q * 128);
                                    f[4 * q] += v.x;
                                    f[4 * q + 1] += v.y;
                                    f[4 * q + 2] += v.z;
                                    f[4 * q + 3] += v.w;
                                }
                            }
                        }
                        float* dst = stage_out + (size_t)row * ostride + 16 * c;
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            *reinterpret_cast<float4*>(dst + 4 * q) = make_float4(f[4 * q], f[4 * q + 1], f[4 * q + 2], f[4 * q + 3]);
                    }
                    epi_bar();
                    // phase 2: coalesced write-out, rows 8w .. 8w+7
                    double* colw = colp + (size_t)warp * p.bn * 2;
                    const int lane_base = 8 * warp;
                    const int nrows = (int)max((int64_t)0, min((int64_t)8, p.n_out - (ms + lane_base)));
                    switch (sel) {
#define S3DSP_WO(idx, OT, RT, SL, ST)                                                                                \
    case idx:                                                                                                        \
        writeout_fast<OT, RT, SL, ST>(p, so_base, ostride, lane_base, lane, ms, n0, limit, nrows, bias4, colw); \
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
                            writeout_generic(p, stage_out, ostride, lane_base, lane, ms, n0, limit, nrows, bias4,
                                             stats ? colw : nullptr);
                    }
                    if (stats) {
                        // deterministic GroupNorm partials of the 128-row tile from the
                        // write-out's per-warp column sums
                        epi_bar();
                        const int64_t t128 = kSub * st + sub;
                        gn_tile_partials<kProdWarps, kEpiThreads>(colp, p.bn, n0, limit, gs, p.gn_groups, tid,
                                                                  p.gn_partials + t128 * p.gn_groups * 2,
                                                                  p.gn_store != 0, epi_bar);
                    }
                    epi_bar();  // the tile and column sums are reused by the next subtile
                }
            }
            // generic-proxy writes to the ring precede the next segment's TMA writes
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            tc_fence_before();
            if (T > 0) acc_ph ^= 1u;
        }
        __syncthreads();
        tc_fence_after();
        if (*abort_flag) break;
    }
    if (warp < kProdWarps) asm volatile("cp.async.wait_all;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(p.tcols) : "memory");
    }
}

size_t sk_smem_bytes(int stages, int bn, int rows) {
    const size_t ring = (size_t)stages * ((size_t)rows * 2 * kKC + (size_t)bn * 2 * kKC);
    const size_t epi = (size_t)128 * (bn + 4) * 4 + colsum_bytes(bn);
    return 1024 /*align slack*/ + (ring > epi ? ring : epi) + (2 * stages + 1) * 8 + 16;
}

}  // namespace

namespace s3dsp {

cudaError_t launch_conv_sk(s3dsp_context* ctx, const s3dsp_kmap* kmap, int kvol, const __nv_bfloat16* in,
                           const __nv_bfloat16* in_b, int cin_a, int64_t n_in, int cin, int in_shift, const __nv_bfloat16* w, const float* bias,
                           const void* residual, uint32_t res_dtype, int res_shift, void* out, uint32_t out_dtype,
                           int64_t n_out, int cout, uint32_t flags, double* gn_partials, int gn_groups, int rows,
                           int csplit, char* error, uint64_t error_capacity, s3d_status* st) {
    *st = S3D_OK;
    (void)n_in;
    if ((rows != 128 && rows != 256) || (csplit != 1 && csplit != 2) || (csplit == 2 && rows != 256)) {
        *st = fail(error, error_capacity, S3D_INTERNAL_ERROR, "stream-K tile rows %d, split %d", rows, csplit);
        return cudaErrorInvalidValue;
    }
    const int cout_pad = (cout + 15) / 16 * 16;
    const int cin_pad = (cin + 63) / 64 * 64;
    const int bn = tc_pick_bn(cout);
    const int nnb = cout_pad / bn;
    const int kchunks = cin_pad / kKC;
    const int64_t tiles = (n_out + 127) / 128;
    const int64_t work_tiles = (n_out + rows - 1) / rows * nnb;
    const int64_t units = work_tiles * kvol;

    int stages = 16;
    while (stages > 2 && sk_smem_bytes(stages, bn, rows) > (size_t)kSmemMax) --stages;
    const size_t smem = sk_smem_bytes(stages, bn, rows);
    if (smem > (size_t)kSmemMax) {
        *st = fail(error, error_capacity, S3D_INTERNAL_ERROR, "conv tile of %d columns does not fit shared memory", bn);
        return cudaErrorInvalidValue;
    }
    // at least ~32 reduction steps (of kKC channels) per CTA before splitting tiles further
    const int64_t min_units = (32 + kchunks - 1) / kchunks;
    int64_t g = (units + min_units - 1) / min_units;
    if (g > ctx->sm_count) g = ctx->sm_count;
    if (g < 1) g = 1;
    if (csplit == 2) {
        // one CTA pair per work tile (the grid may exceed the SM count: pairs then run in waves)
        if (work_tiles > 0x3fffffff) {
            *st = fail(error, error_capacity, S3D_INVALID_ARGUMENT, "too many work tiles for split-K pairs");
            return cudaErrorInvalidValue;
        }
        g = 2 * work_tiles;
    }
    const int grid = (int)g;
    bool split = false;
    for (int i = 1; i < grid && !split && csplit == 1; ++i) split = ((int64_t)i * units / grid) % kvol != 0;

    auto encode = get_encode_fn();
    if (!encode) {
        *st = fail(error, error_capacity, S3D_INTERNAL_ERROR, "cuTensorMapEncodeTiled unavailable");
        return cudaErrorNotSupported;
    }
    const int nb = (bn % 32 == 0) ? 4 : (bn % 16 == 0) ? 2 : 1;
    CUtensorMap wmap;
    {
        const cuuint64_t dims[2] = {(cuuint64_t)cin_pad, (cuuint64_t)kvol * (cuuint64_t)cout_pad};
        const cuuint64_t strides[1] = {(cuuint64_t)cin_pad * 2};
        const cuuint32_t box[2] = {(cuuint32_t)kKC, (cuuint32_t)(bn / nb)};
        const cuuint32_t estr[2] = {1, 1};
        CUresult cr = encode(&wmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (void*)w, dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE,
                             kKC == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (cr != CUDA_SUCCESS) {
            *st = fail(error, error_capacity, S3D_INTERNAL_ERROR, "weight tensor map failed (%d)", (int)cr);
            return cudaErrorInvalidValue;
        }
    }
    uint32_t thalf = 32;
    while ((int)thalf < bn) thalf <<= 1;

    SkParams p;
    p.in = in;
    p.in_b = in_b;
    p.cin_a = in_b ? cin_a : cin;
    p.cin = cin;
    p.in_shift = in_shift;
    p.nbr = kmap ? kmap->nbr : nullptr;
    p.tile_mask = kmap ? kmap->tile_mask : nullptr;
    p.kvol = kvol;
    p.kchunks = kchunks;
    p.cout_pad = cout_pad;
    p.bn = bn;
    p.nb = nb;
    p.stages = stages;
    p.tcols = (uint32_t)(rows / 128) * thalf;
    p.thalf = thalf;
    p.idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(bn >> 3) << 17) | ((128u >> 4) << 24);
    p.bias = bias;
    p.residual = residual;
    p.res_dtype = res_dtype;
    p.res_shift = res_shift;
    p.out = out;
    p.out_dtype = out_dtype;
    p.n_out = n_out;
    p.n_tiles = tiles;
    p.nnb = nnb;
    p.units = units;
    p.grid = grid;
    p.csplit = csplit;
    p.gn_store = nnb == 1;
    p.ws = nullptr;
    p.counters = nullptr;
    p.cout = cout;
    p.flags = flags;
    p.gn_partials = gn_partials;
    p.gn_groups = gn_groups;
    p.status = ctx->d_status;
    p.w = w;
    p.w_bytes = (uint64_t)kvol * (uint64_t)cout_pad * (uint64_t)cin_pad * 2;

    cudaStream_t s = ctx->stream;
    static std::atomic<uint64_t> optin128{0}, optin256{0}, optin128_two{0}, optin256_two{0};
    const bool two = in_b != nullptr;
    auto kernel = rows == 256 ? (two ? conv_sk_kernel<256, true> : conv_sk_kernel<256>)
                              : (two ? conv_sk_kernel<128, true> : conv_sk_kernel<128>);
    cudaError_t e = smem_optin((const void*)kernel, ctx->device,
                               rows == 256 ? (two ? optin256_two : optin256) : (two ? optin128_two : optin128));
    if (e != cudaSuccess) return e;
    if (gn_partials && !p.gn_store) {
        e = cudaMemsetAsync(gn_partials, 0, sizeof(double) * 2 * (size_t)gn_groups * (size_t)tiles, s);
        if (e != cudaSuccess) return e;
    }
    void* ws = nullptr;
    void* counters = nullptr;
    if (split) {
        e = s3dsp::malloc_async(&ws, (size_t)2 * grid * rows * bn * sizeof(float), s);
        if (e == cudaSuccess) e = s3dsp::malloc_async(&counters, (size_t)work_tiles * sizeof(uint32_t), s);
        if (e == cudaSuccess) e = cudaMemsetAsync(counters, 0, (size_t)work_tiles * sizeof(uint32_t), s);
        if (e != cudaSuccess) {
            if (ws) cudaFreeAsync(ws, s);
            if (counters) cudaFreeAsync(counters, s);
            *st = cuda_fail(error, error_capacity, e, "conv workspace");
            return e;
        }
        p.ws = static_cast<float*>(ws);
        p.counters = static_cast<uint32_t*>(counters);
    }
    if (csplit == 2) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)grid);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = s;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 2;
        e = cudaLaunchKernelEx(&cfg, kernel, p, wmap);
        if (e != cudaSuccess) return e;
    } else {
        launch_pdl(kernel, dim3(grid), dim3(kThreads), smem, s, p, wmap);
    }
    e = cudaGetLastError();
    if (ws) cudaFreeAsync(ws, s);
    if (counters) cudaFreeAsync(counters, s);
    return e;
}

}  // namespace s3dsp
