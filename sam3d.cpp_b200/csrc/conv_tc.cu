// Implicit-gather sparse convolution on the 5th-generation tensor cores:
// tcgen05.mma with the f32 accumulator in TMEM; BF16 operands, or f32
// operands as 3xTF32 (kTF32, described at the end of this comment).
//
// Tile: 128 output rows x BN output channels per CTA (BN = a multiple of 16,
// <= 256). The reduction walks (active offset, 64-channel chunk) steps. Per
// step, stage s of a shared-memory ring receives
//   A: the 128 gathered input rows (64 bf16 = 128 B each) by cp.async from
//      512 producer threads (8 threads per row, 16 B each, zero-filled for a
//      missing neighbour); each thread's copies complete onto the stage's
//      mbarrier (cp.async.mbarrier.arrive.noinc), so producers run ahead;
//      a thread reads the kernel-map entries of its own rows itself, one
//      kernel offset ahead of the gathers that use them (no setup pass);
//   B: the BN x 64 weight tile W[o][n0:n0+BN][k0:k0+64] as NB TMA tile loads
//      of BN/NB rows, issued by NB different warps: one thread's TMA ops are
//      serialised (a few hundred cycles each), separate issuers overlap.
// Both use the 128-byte swizzle that the MMA smem descriptors describe. One
// elected thread issues 4 tcgen05.mma (M=128, N=BN, K=16) per step and frees
// the stage with tcgen05.commit.
//
// Epilogue: the accumulator is read back with tcgen05.ld into a padded
// shared-memory tile (warp w: TMEM lanes 32*(w%4).., i.e. its rows, column
// chunks w/4, w/4+4, ...), then written out row by row (warp w: rows
// 8w..8w+7) with coalesced vector loads/stores: bias, residual, GroupNorm
// partial sums (f64) and SiLU are applied on the way. Outputs are written
// once; nothing accumulates through atomics.
//
// Warp roles (672 threads): warps 0-15 gather A and then run the epilogue;
// warps 16-19 issue the weight TMA loads (lane 0 each); warp 20 owns TMEM and
// issues the MMAs.
//
// Every mbarrier wait is bounded (about two seconds of %globaltimer); on
// timeout the CTA records kErrPipelineTimeout, stops issuing work and exits
// through the common teardown, which frees its TMEM.
//
// 3xTF32 (kTF32): f32 operands split into a TF32 high part and its f32
// remainder (input split once per conv, weights at pack time). A 32-channel
// f32 row chunk is the same 128 bytes as a 64-channel bf16 one, so the layout,
// descriptors and TMA boxes are the bf16 ones; a stage holds a high and a low
// half of each operand, and each K step issues lo*hi, hi*lo, hi*hi
// (kind::tf32). The tensor core's f32 accumulation truncates, so each K step
// of a stage has its own TMEM accumulator (two alternating groups for tiles of
// at most 64 columns), summed in f32 by the epilogue.
//
// Replaces the GGML get_rows + mul_mat chains of slat_flow_graph.cpp:112-155
// (SLat conv) and mesh_decoder_graph.cpp:81-103 (mesh conv, per-offset form)
// as one gather-GEMM; in_shift = 3 gathers the parent row of a child, which
// is repeat_children (mesh_decoder_graph.cpp:32-38) without materialising it.
#include "s3dsp_internal.h"
#include "tc_common.cuh"

using namespace s3dsp;
using namespace s3dsp::tc;

namespace {

constexpr int kProdWarps = 16;      // A gather warps (512 threads)
constexpr int kBWarp0 = 16;         // first weight-TMA warp
constexpr int kMaxBWarps = 4;
constexpr int kMmaWarp = 20;
constexpr int kThreads = 21 * 32;
// Each stage's "full" barrier may be split in kFullSplit barriers, one per
// group of producer warps. Measured on B200 (config-2 conv, 85 us with one
// barrier): 4 barriers 115 us, 16 barriers 469 us; one barrier per stage.
constexpr int kFullSplit = 1;

struct TcParams {
    const __nv_bfloat16* in;    // BF16 input [n_in, cin_a]
    const __nv_bfloat16* in_b;  // BF16 second source [n_in, cin - cin_a] (channels [cin_a, cin)) or null
    const float* in_hi;         // 3xTF32: input split into TF32 high parts ...
    const float* in_lo;         // ... and the f32 remainders, [n_in, cin_a] each
    const float* in_hi_b;       // 3xTF32: the second source's parts, [n_in, cin - cin_a] each
    const float* in_lo_b;
    int cin_a;                  // channels read from the first source (== cin for one source)
    int lo_rows;                // 3xTF32: row of the low weight block in the weight tensor map
    int tf_groups;              // 3xTF32: groups of four TMEM accumulators (1, 2, 4 or 8, taken in turn by stage)
    int cin;
    int in_shift;
    const int32_t* nbr;         // [kvol][n_out] or null (identity)
    const uint32_t* tile_mask;  // [tiles] or null
    int kvol;
    int cout_pad;               // packed weight rows per offset
    int bn;
    int nb;                     // weight TMA loads per stage (issuer warps)
    int stages;
    uint32_t idesc;
    const float* bias;
    const void* residual;
    uint32_t res_dtype;
    int res_shift;
    void* out;
    uint32_t out_dtype;
    int64_t n_out;
    int64_t n_tiles;            // 128-row tiles of the output
    int cout;
    uint32_t flags;
    double* gn_partials;
    int gn_store;  // one column tile covers every channel: each slot has one writer
    int gn_groups;
    uint32_t* status;
    const void* w;              // packed weights (for the L2 prefetch before the dependency wait)
    uint64_t w_bytes;
};

// named barrier of the 16 gather/epilogue warps
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 512;" ::: "memory"); }

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
// kPair = false: one CTA per 128-row tile (tcgen05 cta_group::1, M = 128).
// kPair = true: CTA pairs (cluster of 2) share each MMA (cta_group::2,
// M = 256): each CTA gathers its own 128 rows and loads HALF of the weight
// tile, so weight traffic per output row halves. The leader (rank 0) issues
// the MMAs; the peer's weight TMA completes on the leader's barrier and the
// peer's gathered rows are relayed to it by a remote mbarrier arrive.
// kTwo: the input is the channel concat of two sources (p.in_b / p.in_hi_b);
// a separate instance, so the one-source gather keeps its shorter address path
template <bool kPair, int KC, bool kTF32 = false, bool kTwo = false>
__global__ void __launch_bounds__(kThreads, 1)
    conv_tc_kernel(const TcParams p, const __grid_constant__ CUtensorMap wmap) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte aligned base for the swizzled tiles
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int S = p.stages;
    const int brows = kPair ? p.bn / 2 : p.bn;  // weight rows held by this CTA
    // A row chunk: KC elements = 128 bytes (64 bf16, or 32 f32 read as TF32);
    // 3xTF32 stages hold a high and a low half of each operand
    constexpr int kEs = kTF32 ? 4 : 2;        // bytes per element
    constexpr int kRowB = KC * kEs;           // bytes per row chunk
    constexpr int KCB = kRowB / 2;            // the same row in bf16 units (swizzle / descriptors)
    constexpr int kParts = kTF32 ? 2 : 1;
    constexpr int kAHalf = 128 * kRowB;       // bytes of one A half
    constexpr int kAStage = kAHalf * kParts;
    const int bhalf = brows * kRowB;
    const int bstage = bhalf * kParts;
    // layout (offsets from the 1024-aligned base): region0 = max(ring A |
    // ring B, epilogue f32 output tile | f64 GroupNorm column sums), then
    // barriers, tmem holder, abort flag.
    uint8_t* sA = smem;
    uint8_t* sB = smem + (size_t)S * kAStage;
    const size_t ring_bytes = (size_t)S * (kAStage + bstage);
    const size_t epi_bytes = (size_t)128 * (p.bn + 4) * 4 + (size_t)kProdWarps * p.bn * 16;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (ring_bytes > epi_bytes ? ring_bytes : epi_bytes));
    constexpr int kFS = kPair ? 1 : kFullSplit;  // the pair relay arrives on one barrier
    uint64_t* empty = full + S * kFS;
    uint64_t* accum = empty + S;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(accum + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
    float* stage_out = reinterpret_cast<float*>(smem);           // epilogue tile (reuses the ring)
    const int ostride = p.bn + 4;                                 // padded row stride (floats)

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int tile = blockIdx.x;
    const int64_t m0 = (int64_t)tile * 128;
    const int n0 = blockIdx.y * p.bn;

    const uint32_t rank = kPair ? cluster_rank() : 0u;
    const bool leader = rank == 0;
    // 3xTF32 keeps one TMEM accumulator per K step of a stage (and, for tiles of
    // at most 64 columns, a second group used by every other stage), summed in
    // f32 in the epilogue: the tensor core's f32 accumulation truncates, and a
    // fraction of the reduction per accumulator keeps the error inside the F32 gate
    constexpr int kTfStep = kTF32 ? kRowB / 32 : 1;  // accumulators per group: one per K step
    const int tf_groups = kTF32 ? p.tf_groups : 1;
    const int tneed = kTfStep * tf_groups * p.bn;
    const uint32_t tcols = tneed <= 32 ? 32u : (tneed <= 64 ? 64u : (tneed <= 128 ? 128u : (tneed <= 256 ? 256u : 512u)));

    // ---- setup: barriers, TMEM ----
    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            // single CTA: cp.async threads + weight issuers; pair leader: + the
            // peer's relay arrival; pair peer: its own cp.async threads only
            for (int j = 0; j < kFS; ++j) {
                uint32_t cnt = kProdWarps * 32 / kFS;
                if (j == 0) cnt += !kPair ? p.nb : leader ? p.nb + 1 : 0;
                mbar_init(smem_u32(full + s * kFS + j), cnt);
            }
            mbar_init(smem_u32(empty + s), 1);
        }
        mbar_init(smem_u32(accum), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        if (kPair) {
            asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                         "r"(tcols)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
        } else {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                         "r"(tcols)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        }
    }
    // the weights do not depend on the previous kernel: start bringing this
    // CTA's share into L2 while it finishes
    if (tid == 32)
        prefetch_share_l2(p.w, p.w_bytes, blockIdx.y * gridDim.x + blockIdx.x, gridDim.x * gridDim.y);
    if (warp == 2) prefetch_lines_l2(p.bias, (uint64_t)p.cout * 4, lane);  // read by the epilogue
    tc_fence_before();
    __syncthreads();
    if (kPair) cluster_sync();  // the peer's barriers exist before any remote arrive
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    // everything above touched shared memory, TMEM, parameters and the L2 hint only
    pdl_wait();
    pdl_trigger();
    // both CTAs of a pair walk the union of their tiles' active offsets
    uint32_t mask = 1u;
    if (p.nbr) {
        mask = 0x7ffffffu;
        if (p.tile_mask) {
            mask = tile < p.n_tiles ? p.tile_mask[tile] : 0u;
            if (kPair && (tile ^ 1) < p.n_tiles) mask |= p.tile_mask[tile ^ 1];
        }
    }
    mask &= (p.kvol >= 32) ? 0xffffffffu : ((1u << p.kvol) - 1u);
    // KC-channel reduction chunks per offset
    const int kchunks = kTF32 ? (p.cin + KC - 1) / KC : (p.cin + 63) / 64 * (64 / KC);
    const int T = __popc(mask) * kchunks;

    bool prod_ok = true;
    if (warp < kProdWarps) {
        // ================= A producers: cp.async gathers =================
        // Each thread gathers fixed rows (rg + kRowStep * i) and reads their map
        // entries itself, one kernel offset ahead of the gathers that use them.
        constexpr int kCpr = kRowB / 16;      // 16-byte chunks per row
        constexpr int kRowStep = 512 / kCpr;  // rows covered by one pass of the 512 threads
        constexpr int kMine = 128 / kRowStep;
        const int c16 = tid & (kCpr - 1);
        const int rg = tid / kCpr;  // rows rg, rg + kRowStep, ...
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
        for (int it = 0; it < T; ++it) {
            const int s = it % S;
            const uint32_t ph = (uint32_t)(it / S) & 1u;
            const int kc = it % kchunks;
            if (kc == 0) {
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
            const int k0 = kc * KC + c16 * (16 / kEs);
            const uint32_t a_base = smem_u32(sA + (size_t)s * kAStage);
            if constexpr (kTwo) {
                // channel concat of two sources: the source holding channel k0, its
                // row stride and column, fixed for the whole stage
                const bool kin = k0 < p.cin;
                const bool from_a = k0 < p.cin_a;
                const int64_t ld = from_a ? p.cin_a : p.cin - p.cin_a;
                const int kk = from_a ? k0 : k0 - p.cin_a;
#pragma unroll
                for (int i = 0; i < kMine; ++i) {
                    const int row = rg + kRowStep * i;
                    const int32_t src = cur[i];
                    const bool valid = kin && src >= 0;
                    // an invalid copy reads nothing; it keeps the first source's base address
                    const int64_t off = valid ? (int64_t)src * ld + kk : 0;
                    const uint32_t d = a_base + row * kRowB + ((c16 ^ kmajor_swz<KCB>(row)) << 4);
                    if constexpr (kTF32) {
                        cp_async_16(d, (valid && !from_a ? p.in_hi_b : p.in_hi) + off, valid ? 16u : 0u);
                        cp_async_16(d + kAHalf, (valid && !from_a ? p.in_lo_b : p.in_lo) + off, valid ? 16u : 0u);
                    } else {
                        cp_async_16(d, (valid && !from_a ? p.in_b : p.in) + off, valid ? 16u : 0u);
                    }
                }
            } else {
#pragma unroll
                for (int i = 0; i < kMine; ++i) {
                    const int row = rg + kRowStep * i;
                    const int32_t src = cur[i];
                    const bool valid = src >= 0 && k0 < p.cin;
                    const uint32_t d = a_base + row * kRowB + ((c16 ^ kmajor_swz<KCB>(row)) << 4);
                    if constexpr (kTF32) {
                        const int64_t off = valid ? (int64_t)src * p.cin + k0 : 0;
                        cp_async_16(d, p.in_hi + off, valid ? 16u : 0u);
                        cp_async_16(d + kAHalf, p.in_lo + off, valid ? 16u : 0u);
                    } else {
                        const void* g = valid ? (const void*)(p.in + (int64_t)src * p.cin + k0) : (const void*)p.in;
                        cp_async_16(d, g, valid ? 16u : 0u);
                    }
                }
            }
            cp_async_arrive_noinc(smem_u32(full + s * kFS + warp / (kProdWarps / kFS)));
        }
        if (p.residual && tile < p.n_tiles) {
            // the epilogue reads this tile's residual rows: start bringing them
            // into L2 now, while the last stages are still in flight
            const int esz = p.res_dtype == S3DSP_F32 ? 4 : 2;
            const int64_t r = m0 + (tid >> 2);
            const int len = min(p.bn, p.cout - n0) * esz;
            if (r < p.n_out) {
                const char* row = static_cast<const char*>(p.residual) +
                                  (((r >> p.res_shift) * p.cout + n0) * (int64_t)esz);
                for (int b = (tid & 3) * 128; b < len; b += 4 * 128)
                    asm volatile("prefetch.global.L2 [%0];" ::"l"(row + b));
            }
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
    } else if (warp < kBWarp0 + kMaxBWarps) {
        // ================= weight TMA issuers =================
        const int j = warp - kBWarp0;
        if (lane == 0 && j < p.nb) {
            uint32_t mrem = mask;
            int o = 0;
            const int rows = brows / p.nb;
            const uint32_t bytes = (uint32_t)rows * kRowB;
            for (int it = 0; it < T; ++it) {
                const int s = it % S;
                const uint32_t ph = (uint32_t)(it / S) & 1u;
                const int kc = it % kchunks;
                if (kc == 0) {
                    o = __ffs(mrem) - 1;
                    mrem &= mrem - 1;
                }
                if (!mbar_wait(smem_u32(empty + s), ph ^ 1u, abort_flag, p.status)) break;
                const uint32_t fb = smem_u32(full + s * kFS);
                const uint32_t dst = smem_u32(sB + (size_t)s * bstage + (size_t)j * rows * kRowB);
                const int y = o * p.cout_pad + n0 + (int)rank * brows + j * rows;
                if (!kPair) {
                    mbar_arrive_tx(fb, bytes * kParts);
                    tma_load_2d(dst, &wmap, kc * KC, y, fb);
                    if (kTF32) tma_load_2d(dst + bhalf, &wmap, kc * KC, y + p.lo_rows, fb);
                } else {
                    // the leader expects both CTAs' slice j; both complete on its barrier
                    if (leader) mbar_arrive_tx(fb, 2 * bytes);
                    tma_load_2d_pair(dst, &wmap, kc * KC, y, map_to_rank(fb, 0));
                }
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0 && kPair && !leader) {
            // ================= relay (pair peer): gathered rows landed -> leader =================
            for (int it = 0; it < T; ++it) {
                const int s = it % S;
                const uint32_t ph = (uint32_t)(it / S) & 1u;
                if (!mbar_wait(smem_u32(full + s * kFS), ph, abort_flag, p.status)) break;
                // the rows were written through the generic proxy; the leader's
                // tensor core reads them through the async proxy
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_arrive_remote(map_to_rank(smem_u32(full + s * kFS), 0));
            }
        } else if (lane == 0) {
            // ================= MMA issuer =================
            bool ok = true;
            for (int it = 0; it < T; ++it) {
                const int s = it % S;
                const uint32_t ph = (uint32_t)(it / S) & 1u;
                bool got = true;
                for (int j = 0; j < kFS && got; ++j)
                    got = kPair ? mbar_wait_cluster(smem_u32(full + s * kFS + j), ph, abort_flag, p.status)
                                : mbar_wait(smem_u32(full + s * kFS + j), ph, abort_flag, p.status);
                if (!got) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a0 = smem_u32(sA + (size_t)s * kAStage);
                const uint32_t b0 = smem_u32(sB + (size_t)s * bstage);
                if (kPair) {
#pragma unroll
                    for (int k = 0; k < kRowB / 32; ++k)
                        mma_bf16_pair(tmem, kmajor_desc<KCB>(a0 + 32 * k), kmajor_desc<KCB>(b0 + 32 * k), p.idesc,
                                      (it > 0 || k > 0) ? 1u : 0u);
                    mma_commit_pair(smem_u32(empty + s));                       // this CTA's stage
                    mma_commit_pair(map_to_rank(smem_u32(empty + s), 1));      // the peer's stage
                } else {
#pragma unroll
                    for (int k = 0; k < kRowB / 32; ++k) {
                        if constexpr (kTF32) {
                            // 3xTF32: lo*hi + hi*lo + hi*hi (small products first) into the
                            // accumulator of K step k
                            const uint64_t ah = kmajor_desc<KCB>(a0 + 32 * k), al = kmajor_desc<KCB>(a0 + kAHalf + 32 * k);
                            const uint64_t bh = kmajor_desc<KCB>(b0 + 32 * k), bl = kmajor_desc<KCB>(b0 + bhalf + 32 * k);
                            const int grp = it % tf_groups;
                            const uint32_t dk = tmem + (uint32_t)((grp * kTfStep + k) * p.bn);
                            mma_tf32(dk, al, bh, p.idesc, it >= tf_groups ? 1u : 0u);
                            mma_tf32(dk, ah, bl, p.idesc, 1u);
                            mma_tf32(dk, ah, bh, p.idesc, 1u);
                        } else {
                            mma_bf16(tmem, kmajor_desc<KCB>(a0 + 32 * k), kmajor_desc<KCB>(b0 + 32 * k), p.idesc,
                                     (it > 0 || k > 0) ? 1u : 0u);
                        }
                    }
                    mma_commit(smem_u32(empty + s));
                }
            }
            if (ok && T > 0) {
                if (kPair) {
                    mma_commit_pair(smem_u32(accum));
                    mma_commit_pair(map_to_rank(smem_u32(accum), 1));
                } else {
                    mma_commit(smem_u32(accum));
                }
            }
        }
        __syncwarp();
    }
    if (warp < kProdWarps) {
        // ================= epilogue (all 16 gather warps, after their gathers) =================
        bool have_acc = T > 0 && prod_ok && mbar_wait(smem_u32(accum), 0, abort_flag, p.status);
        have_acc = __all_sync(0xffffffffu, have_acc);
        tc_fence_after();
        // phase 1: TMEM -> padded smem tile. Warp w reads TMEM lanes 32*(w%4)..
        // (its rows), 16-column chunks w/4, w/4 + 4, ...
        {
            const int lq = warp & 3;
            float* dst = stage_out + (size_t)(32 * lq + lane) * ostride;
            const uint32_t taddr = tmem + ((uint32_t)(32 * lq) << 16);
            for (int c0 = 16 * (warp >> 2); c0 < p.bn; c0 += 64) {
                float f[16];
                if (have_acc) {
                    tmem_ld16(taddr + (uint32_t)c0, f);
                    // 3xTF32: the other accumulators that were written, summed in order in f32
                    const int n_acc = kTfStep * (T < tf_groups ? T : tf_groups);
                    for (int a = 1; a < n_acc; ++a) {
                        float g[16];
                        tmem_ld16(taddr + (uint32_t)(a * p.bn + c0), g);
#pragma unroll
                        for (int j = 0; j < 16; ++j) f[j] += g[j];
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) f[j] = 0.f;
                }
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    *reinterpret_cast<float4*>(dst + c0 + 4 * q) = make_float4(f[4 * q], f[4 * q + 1], f[4 * q + 2], f[4 * q + 3]);
            }
        }
        epi_bar();
        // phase 2: bias / residual / SiLU / GroupNorm partials on the way out
        tile_writeout<kProdWarps>(p, smem, ostride, warp, lane, tid, m0, n0,
                                  p.gn_partials && tile < p.n_tiles ? p.gn_partials + (int64_t)tile * p.gn_groups * 2 : nullptr,
                                  epi_bar);
        tc_fence_before();
    }

    __syncthreads();
    if (kPair) cluster_sync();  // no CTA leaves while its pair may still touch its smem/TMEM
    if (warp == kMmaWarp) {
        tc_fence_after();
        if (kPair)
            asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tcols) : "memory");
        else
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tcols) : "memory");
    }
}

// stage = 128 gathered rows + brows weight rows, 128 bytes each, per part
// (3xTF32: a high and a low part)
size_t stage_bytes(int brows, int parts) { return (size_t)(128 + brows) * 128 * parts; }
size_t smem_bytes(int stages, int brows, int parts, int bn) {
    const size_t ring = (size_t)stages * stage_bytes(brows, parts);
    const size_t epi = (size_t)128 * (bn + 4) * 4 + (size_t)kProdWarps * bn * 16;
    return 1024 /*align slack*/ + (ring > epi ? ring : epi) + ((kFullSplit + 1) * stages + 1) * 8 + 16;
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

// One launcher for both tensor-core modes: BF16 (in = bf16 rows) and 3xTF32
// (in = high parts, in_lo = remainders, both f32; weights packed as a high
// block followed by a low block).
static cudaError_t launch_tc_impl(s3dsp_context* ctx, const s3dsp_kmap* kmap, int kvol, const void* in, const float* in_lo,
                           const void* in_b, const float* in_lo_b, int cin_a, int cin, int in_shift, const void* w, const float* bias, const void* residual,
                           uint32_t res_dtype, int res_shift, void* out, uint32_t out_dtype, int64_t n_out, int cout,
                           uint32_t flags, double* gn_partials, int gn_groups, char* error, uint64_t error_capacity,
                           s3d_status* st) {
    *st = S3D_OK;
    const bool tf32 = in_lo != nullptr;
    const int cout_pad = (cout + 15) / 16 * 16;
    const int cin_pad = tf32 ? (cin + 31) / 32 * 32 : (cin + 63) / 64 * 64;
    int bn = tc_pick_bn(cout);
    // 3xTF32: two-part stages (at most 128 columns keeps three stages), and
    // TMEM for 4 accumulators per group. The tensor core's f32 accumulation
    // truncates once per MMA, so the error grows with the products each
    // accumulator takes: longer reductions take narrower tiles and more
    // groups (tile columns x 4 x groups = 512 TMEM columns), i.e. at most
    // about 1,100-1,700 products per accumulator for the 1024- and 2048-wide
    // SLat layers (27 x 1024 and 27 x 2048)
    const int64_t kred = (int64_t)cin * kvol;
    const int tf_cap = kred > 32768 ? 16 : kred > 16384 ? 32 : kred > 4096 ? 64 : 128;
    if (tf32 && bn > tf_cap) {
        bn = 16;
        for (int c = tf_cap; c >= 16; c -= 16)
            if (cout_pad % c == 0) {
                bn = c;
                break;
            }
    }
    const int64_t tiles = (n_out + 127) / 128;
    // CTA pairs need an even row-tile count (the last pair may hold one empty tile)
    // CTA pairs read one source; a concat runs on the one-CTA kernel
    const bool pair = !tf32 && !in_b && (flags & S3DSP_CONV_CTA_PAIR) != 0;
    const int brows = pair ? bn / 2 : bn;
    const int parts = tf32 ? 2 : 1;
    // 128-byte row chunks per stage (64 bf16 / 32 f32): 64-byte bf16 stages
    // (twice as many for the same shared memory) measured slower on B200
    // (config-2 conv 119-123 us vs 81-85 us): a stage has a fixed cost beyond its bytes
    const int kc = tf32 ? 32 : 64;
    int stages = (int)((200 * 1024) / stage_bytes(brows, parts));
    if (stages > 16) stages = 16;

    auto encode = get_encode_fn();
    if (!encode) {
        *st = fail(error, error_capacity, S3D_INTERNAL_ERROR, "cuTensorMapEncodeTiled unavailable");
        return cudaErrorNotSupported;
    }
    // weight tile rows per TMA load: NB issuers, slices a multiple of 8 rows
    const int nb = (brows % 32 == 0) ? 4 : (brows % 16 == 0) ? 2 : 1;
    CUtensorMap wmap;
    {
        const int es = tf32 ? 4 : 2;
        const cuuint64_t dims[2] = {(cuuint64_t)cin_pad, (cuuint64_t)parts * kvol * (cuuint64_t)cout_pad};
        const cuuint64_t strides[1] = {(cuuint64_t)cin_pad * es};
        const cuuint32_t box[2] = {(cuuint32_t)kc, (cuuint32_t)(brows / nb)};
        const cuuint32_t estr[2] = {1, 1};
        CUresult cr = encode(&wmap, tf32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                             const_cast<void*>(w), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (cr != CUDA_SUCCESS) {
            *st = fail(error, error_capacity, S3D_INTERNAL_ERROR, "weight tensor map failed (%d)", (int)cr);
            return cudaErrorInvalidValue;
        }
    }
    TcParams p;
    p.in = tf32 ? nullptr : static_cast<const __nv_bfloat16*>(in);
    p.in_b = tf32 ? nullptr : static_cast<const __nv_bfloat16*>(in_b);
    p.in_hi = tf32 ? static_cast<const float*>(in) : nullptr;
    p.in_lo = in_lo;
    p.in_hi_b = tf32 ? static_cast<const float*>(in_b) : nullptr;
    p.in_lo_b = in_lo_b;
    p.cin_a = in_b ? cin_a : cin;
    p.lo_rows = kvol * cout_pad;
    p.tf_groups = tf32 ? (bn <= 16 ? 8 : bn <= 32 ? 4 : bn <= 64 ? 2 : 1) : 1;
    p.cin = cin;
    p.in_shift = in_shift;
    p.nbr = kmap ? kmap->nbr : nullptr;
    p.tile_mask = kmap ? kmap->tile_mask : nullptr;
    p.kvol = kvol;
    p.cout_pad = cout_pad;
    p.bn = bn;
    p.nb = nb;
    p.stages = stages;
    const uint32_t mma_m = pair ? 256u : 128u;  // pair: M spans both CTAs' rows
    // instruction descriptor: f32 accumulator; A, B = BF16 (1) or TF32 (2), both K-major
    const uint32_t fmt = tf32 ? 2u : 1u;
    p.idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(bn >> 3) << 17) | ((mma_m >> 4) << 24);
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
    p.gn_groups = gn_groups;
    p.gn_store = cout_pad == bn;
    p.status = ctx->d_status;
    p.w = w;
    p.w_bytes = (uint64_t)parts * kvol * (uint64_t)cout_pad * (uint64_t)cin_pad * (tf32 ? 4 : 2);

    const size_t smem = smem_bytes(stages, brows, parts, bn);
    static std::atomic<uint64_t> optin_pair{0}, optin_single{0}, optin_tf32{0};
    const bool two = in_b != nullptr;
    static std::atomic<uint64_t> optin_tf32_two{0}, optin_single_two{0};
    cudaError_t e = tf32 ? (two ? smem_optin((const void*)conv_tc_kernel<false, 32, true, true>, ctx->device,
                                             optin_tf32_two)
                                : smem_optin((const void*)conv_tc_kernel<false, 32, true>, ctx->device, optin_tf32))
                    : pair ? smem_optin((const void*)conv_tc_kernel<true, 64>, ctx->device, optin_pair)
                           : (two ? smem_optin((const void*)conv_tc_kernel<false, 64, false, true>, ctx->device,
                                               optin_single_two)
                                  : smem_optin((const void*)conv_tc_kernel<false, 64>, ctx->device, optin_single));
    if (e == cudaSuccess && smem > (size_t)kSmemOptIn) e = cudaErrorInvalidValue;
    if (e != cudaSuccess) return e;
    if (gn_partials && !p.gn_store) {
        e = cudaMemsetAsync(gn_partials, 0, sizeof(double) * 2 * (size_t)gn_groups * (size_t)tiles, ctx->stream);
        if (e != cudaSuccess) return e;
    }
    if (!pair) {
        const dim3 grid((unsigned)tiles, (unsigned)(cout_pad / bn));
        if (tf32)
            e = two ? launch_pdl(conv_tc_kernel<false, 32, true, true>, grid, dim3(kThreads), smem, ctx->stream, p, wmap)
                    : launch_pdl(conv_tc_kernel<false, 32, true>, grid, dim3(kThreads), smem, ctx->stream, p, wmap);
        else
            e = two ? launch_pdl(conv_tc_kernel<false, 64, false, true>, grid, dim3(kThreads), smem, ctx->stream, p,
                                 wmap)
                    : launch_pdl(conv_tc_kernel<false, 64>, grid, dim3(kThreads), smem, ctx->stream, p, wmap);
        if (e != cudaSuccess) return e;
        return cudaGetLastError();
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((tiles + 1) / 2 * 2), (unsigned)(cout_pad / bn));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, conv_tc_kernel<true, 64>, p, wmap);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

cudaError_t launch_conv_tc(s3dsp_context* ctx, const s3dsp_kmap* kmap, int kvol,
                           const __nv_bfloat16* in, const __nv_bfloat16* in_b, int cin_a, int64_t n_in, int cin,
                           int in_shift, const __nv_bfloat16* w, const float* bias, const void* residual,
                           uint32_t res_dtype, int res_shift, void* out, uint32_t out_dtype,
                           int64_t n_out, int cout, uint32_t flags, double* gn_partials,
                           int gn_groups, char* error, uint64_t error_capacity, s3d_status* st) {
    (void)n_in;
    return launch_tc_impl(ctx, kmap, kvol, in, nullptr, in_b, nullptr, cin_a, cin, in_shift, w, bias, residual,
                          res_dtype, res_shift, out, out_dtype, n_out, cout, flags, gn_partials, gn_groups, error,
                          error_capacity, st);
}

cudaError_t launch_conv_tf32x3(s3dsp_context* ctx, const s3dsp_kmap* kmap, int kvol, const float* in_hi,
                               const float* in_lo, const float* in_hi_b, const float* in_lo_b, int cin_a, int cin,
                               int in_shift, const float* w, const float* bias,
                               const void* residual, uint32_t res_dtype, int res_shift, void* out, uint32_t out_dtype,
                               int64_t n_out, int cout, uint32_t flags, double* gn_partials, int gn_groups,
                               char* error, uint64_t error_capacity, s3d_status* st) {
    return launch_tc_impl(ctx, kmap, kvol, in_hi, in_lo, in_hi_b, in_lo_b, cin_a, cin, in_shift, w, bias, residual,
                          res_dtype, res_shift, out, out_dtype, n_out, cout, flags, gn_partials, gn_groups, error,
                          error_capacity, st);
}

}  // namespace s3dsp
