// Coordinate hash and kernel-map construction.
//
// Hash: open addressing with linear probing over a power-of-two table of
// 16-byte slots {64-bit packed key, first row} (load factor <= 1/4). The row
// is the FIRST row of each key (atomicMin), which reproduces the
// std::map::emplace "first insert wins" rule of SlatTables::build
// (src/objects_runtime/sparse_ops.cpp:119-124). Coordinates are read as one
// int4 per row (coalesced 16-byte loads) and a probe is one 16-byte load that
// returns key and row together. Every probe loop is bounded by the table
// size.
//
// Kernel maps are stored offset-major, nbr[o * n_out + r] (-1 = none), so the
// conv's gather loader reads 128 consecutive output rows of one offset with
// one coalesced 512-byte load, and a per-128-row-tile bitmask records which
// offsets have any neighbour (the conv skips empty offsets).
#include "s3dsp_internal.h"
#include "hash_view.cuh"

#include <mutex>

using namespace s3dsp;
using namespace s3dsp::hash;

namespace {

// every slot empty: key all-ones, row INT32_MAX (the atomicMin identity)
__global__ void hash_init_kernel(ulonglong2* __restrict__ slots, uint64_t cap) {
    pdl_wait();
    pdl_trigger();
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < cap; i += (uint64_t)gridDim.x * blockDim.x)
        slots[i] = make_ulonglong2(kEmptyKey, 0x7fffffffull);
}

// inserts row i and keeps a copy of its coordinates in the hash
__global__ void hash_insert_kernel(const int4* __restrict__ coords, int64_t n, int4* __restrict__ own,
                                   ulonglong2* slots, unsigned long long mask, int32_t reject_dups,
                                   uint32_t* status) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int4 c = coords[i];
        own[i] = c;
        unsigned long long key;
        if (!pack_key(c.x, c.y, c.z, c.w, key)) {
            atomicOr(status, kErrCoordRange);
            continue;
        }
        unsigned long long s = mix64(key) & mask;
        bool placed = false;
        for (unsigned long long p = 0; p <= mask; ++p) {
            unsigned long long* kp = reinterpret_cast<unsigned long long*>(slots + s);
            const unsigned long long prev = atomicCAS(kp, kEmptyKey, key);
            if (prev == kEmptyKey || prev == key) {
                atomicMin(reinterpret_cast<int*>(kp + 1), (int)i);  // low half of the row word
                if (prev == key) {
                    atomicAdd(status + 1, 1u);
                    if (reject_dups) atomicOr(status, kErrDuplicate);
                }
                placed = true;
                break;
            }
            s = (s + 1) & mask;
        }
        if (!placed) atomicOr(status, kErrHashFull);
    }
}

// first row holding each row's key (a duplicate row is not its own first row)
__global__ void hash_self_kernel(const int4* __restrict__ coords, int64_t n, HashView h,
                                 int32_t* __restrict__ self_row) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int4 c = coords[i];
        self_row[i] = h.find_coord(c.x, c.y, c.z, c.w);
    }
}

__global__ void hash_lookup_kernel(const int4* __restrict__ q, int64_t m, HashView h,
                                   int32_t* __restrict__ rows) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < m;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int4 c = q[i];
        rows[i] = h.find_coord(c.x, c.y, c.z, c.w);
    }
}

// Submanifold 3x3x3 map, offset-major. One block per 128-row tile; thread
// (slab s, row r), s = threadIdx.x / 128, owns the nine offsets with
// dx = s - 1 (o = 9 s .. 9 s + 8, o = kd * 9 + kh * 3 + kw as in
// sparse_ops.cpp:132) of row r. Its nine probes are issued back to back, a
// warp's stores nbr[o * n + r] are coalesced, and the block writes its
// tile's 27-bit offset mask with one plain store (no zeroing pass, no global
// atomics). A duplicate row (not the first holding its key) gets no
// neighbours, as SlatTables::build iterates the unique map entries
// (sparse_ops.cpp:129-139). The first row comes from the hash's self-row
// array when the table is larger than L2 can serve (one probe per row, done
// once), else from a probe of the row's own key.
__device__ __forceinline__ int32_t probe_rest(const HashView& h, unsigned long long key, unsigned long long slot) {
    for (unsigned long long p = 1; p <= h.mask; ++p) {
        slot = (slot + 1) & h.mask;
        const ulonglong2 q = __ldg(h.slots + slot);
        if (q.x == key) return (int32_t)(uint32_t)q.y;
        if (q.x == kEmptyKey) return -1;
    }
    return -1;
}

constexpr int kSlabs = 3;  // dx = -1, 0, +1

// Output row r is hash row row0 + r (r < n).
__global__ void __launch_bounds__(kTileRows * kSlabs) kmap_subm3_kernel(const int4* __restrict__ coords, int64_t row0,
                                                                        int64_t n, HashView h,
                                                                        const int32_t* __restrict__ self_row,
                                                                        int32_t* __restrict__ nbr,
                                                                        uint32_t* __restrict__ tile_mask) {
    pdl_wait();
    pdl_trigger();
    const int s = threadIdx.x / kTileRows;
    const int dx = s - 1;
    const int64_t r = (int64_t)blockIdx.x * kTileRows + threadIdx.x % kTileRows;
    __shared__ uint32_t block_bits;
    if (threadIdx.x == 0) block_bits = 0;
    __syncthreads();
    uint32_t bits = 0;
    if (r < n) {
        const int64_t hr = row0 + r;  // the row in the hash
        const int4 c = __ldg(coords + hr);
        int32_t self = -1;
        if (self_row) {
            self = __ldg(self_row + hr);
        } else {
            unsigned long long ks;
            if (pack_key(c.x, c.y, c.z, c.w, ks)) {
                const unsigned long long ss = mix64(ks) & h.mask;
                const ulonglong2 qs = __ldg(h.slots + ss);
                if (qs.x == ks) self = (int32_t)(uint32_t)qs.y;
                else if (qs.x != kEmptyKey) self = probe_rest(h, ks, ss);
            }
        }
        const bool first = self == (int32_t)hr;
        unsigned long long key[9], slot[9];
        ulonglong2 q[9];
        bool ok[9];
#pragma unroll
        for (int j = 0; j < 9; ++j) {
            ok[j] = first && pack_key(c.x, c.y + dx, c.z + j / 3 - 1, c.w + j % 3 - 1, key[j]);
            slot[j] = ok[j] ? (mix64(key[j]) & h.mask) : 0;
            q[j] = ok[j] ? __ldg(h.slots + slot[j]) : make_ulonglong2(kEmptyKey, 0);
        }
#pragma unroll
        for (int j = 0; j < 9; ++j) {
            int32_t res = -1;
            if (ok[j]) {
                if (q[j].x == key[j]) res = (int32_t)(uint32_t)q[j].y;
                else if (q[j].x != kEmptyKey) res = probe_rest(h, key[j], slot[j]);
            }
            nbr[(int64_t)(9 * s + j) * n + r] = res;
            if (res >= 0) bits |= 1u << (9 * s + j);
        }
    }
    bits = __reduce_or_sync(0xffffffffu, bits);
    if ((threadIdx.x & 31) == 0 && bits) atomicOr(&block_bits, bits);
    __syncthreads();
    if (threadIdx.x == 0) tile_mask[blockIdx.x] = block_bits;
}

// Child geometry of MeshSubdivideTables (sparse_ops.cpp:346-365): for child
// bits j and offset o, which of the parent's 27 neighbours holds the target
// child, and which of its 8 children it is.
// Child-adjacency tables of the subdivide map, fixed at compile time: for child
// j (bits xb,yb,zb) and offset o (d = (o/9-1, (o/3)%3-1, o%3-1)), t = bit + d
// per axis in [-1, 2]; the neighbour's parent is offset floor(t/2) from the
// child's parent (par) and the neighbour is that parent's child t mod 2 (chl).
struct AdjTables {
    uint8_t par[8][27];
    uint8_t chl[8][27];
};
constexpr AdjTables make_adjacency() {
    AdjTables t{};
    for (int j = 0; j < 8; ++j) {
        const int bits[3] = {j >> 2, (j >> 1) & 1, j & 1};
        for (int o = 0; o < 27; ++o) {
            const int d[3] = {o / 9 - 1, (o / 3) % 3 - 1, o % 3 - 1};
            int pd[3] = {0, 0, 0}, tb[3] = {0, 0, 0};
            for (int a = 0; a < 3; ++a) {
                const int v = bits[a] + d[a];
                pd[a] = v < 0 ? -1 : (v > 1 ? 1 : 0);
                tb[a] = v - 2 * pd[a];
            }
            t.par[j][o] = (uint8_t)((pd[0] + 1) * 9 + (pd[1] + 1) * 3 + (pd[2] + 1));
            t.chl[j][o] = (uint8_t)(tb[0] * 4 + tb[1] * 2 + tb[2]);
        }
    }
    return t;
}
__constant__ AdjTables c_adj = make_adjacency();

// One block = 32 parents = 256 children. Phase 1: 27 probes per parent into
// shared memory. Phase 2: 27 x 256 child entries written offset-major
// (coalesced), child coords written as int4.
__global__ void __launch_bounds__(256) subdivide_kernel(const int4* __restrict__ parents, int64_t np,
                                                        HashView h, int4* __restrict__ child_coords,
                                                        int32_t* __restrict__ nbr,
                                                        uint32_t* __restrict__ tile_mask) {
    pdl_wait();
    pdl_trigger();
    __shared__ int32_t padj[32][28];
    const int64_t p0 = (int64_t)blockIdx.x * 32;
    for (int t = threadIdx.x; t < 32 * 27; t += blockDim.x) {
        const int pl = t / 27, o = t % 27;
        const int64_t p = p0 + pl;
        int32_t res = -1;
        if (p < np) {
            const int4 c = parents[p];
            res = h.find_coord(c.x, c.y + o / 9 - 1, c.z + (o / 3) % 3 - 1, c.w + o % 3 - 1);
        }
        padj[pl][o] = res;
    }
    const int c = threadIdx.x;
    const int pl = c >> 3, j = c & 7;
    const int64_t p = p0 + pl;
    const int64_t nc = np * 8;
    const int64_t child = p0 * 8 + c;
    if (p < np) {
        const int4 pc = parents[p];
        child_coords[child] = make_int4(pc.x, pc.y * 2 + (j >> 2), pc.z * 2 + ((j >> 1) & 1), pc.w * 2 + (j & 1));
    }
    __syncthreads();
    for (int o = 0; o < 27; ++o) {
        int32_t v = -1;
        if (p < np) {
            const int32_t tp = padj[pl][c_adj.par[j][o]];
            if (tp >= 0) v = tp * 8 + c_adj.chl[j][o];
            nbr[o * nc + child] = v;
        }
        const unsigned any = __ballot_sync(0xffffffffu, v >= 0);
        if ((c & 31) == 0 && any) atomicOr(tile_mask + (child / kTileRows), 1u << o);
    }
}

__global__ void export_dense_kernel(const int32_t* __restrict__ nbr, int64_t n, int32_t kvol,
                                    int32_t sentinel, int32_t* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n * 27;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / 27;
        const int o = (int)(i - r * 27);
        int32_t v = o < kvol ? nbr[o * n + r] : -1;
        out[i] = v < 0 ? sentinel : v;
    }
}

// pair lists: counts per (offset, block) -> exclusive scan -> scatter
constexpr int kPairBlock = 1024;

__global__ void pair_count_kernel(const int32_t* __restrict__ nbr, int64_t n, int32_t* counts,
                                  int64_t nblk) {
    pdl_wait();
    pdl_trigger();
    const int o = blockIdx.y;
    const int64_t r = blockIdx.x * (int64_t)kPairBlock + threadIdx.x;
    const int valid = (r < n) && nbr[o * n + r] >= 0;
    const int c = __syncthreads_count(valid);
    if (threadIdx.x == 0) counts[o * nblk + blockIdx.x] = c;
}

// single-block exclusive scan of m ints into int64 starts (m is small:
// 27 * ceil(n / 1024))
__global__ void pair_scan_kernel(const int32_t* counts, int64_t m, int64_t* starts) {
    pdl_wait();
    pdl_trigger();
    __shared__ int64_t carry;
    __shared__ int64_t warp_sums[32];
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int64_t base = 0; base < m; base += blockDim.x) {
        const int64_t i = base + threadIdx.x;
        int64_t v = i < m ? counts[i] : 0;
        // inclusive warp scan
        const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
        for (int d = 1; d < 32; d <<= 1) {
            const int64_t t = __shfl_up_sync(0xffffffffu, v, d);
            if (lane >= d) v += t;
        }
        if (lane == 31) warp_sums[w] = v;
        __syncthreads();
        if (w == 0) {
            int64_t s = lane < (int)(blockDim.x >> 5) ? warp_sums[lane] : 0;
            for (int d = 1; d < 32; d <<= 1) {
                const int64_t t = __shfl_up_sync(0xffffffffu, s, d);
                if (lane >= d) s += t;
            }
            warp_sums[lane] = s;
        }
        __syncthreads();
        const int64_t incl = v + (w > 0 ? warp_sums[w - 1] : 0);
        const int64_t excl = incl - (i < m ? counts[i] : 0);
        if (i < m) starts[i] = carry + excl;
        __syncthreads();
        if (threadIdx.x == blockDim.x - 1) carry += incl;
        __syncthreads();
    }
    if (threadIdx.x == 0) starts[m] = carry;
}

__global__ void pair_write_kernel(const int32_t* __restrict__ nbr, int64_t n, const int64_t* starts,
                                  int64_t nblk, int32_t* __restrict__ pin, int32_t* __restrict__ pout) {
    pdl_wait();
    pdl_trigger();
    __shared__ int warp_cnt[kPairBlock / 32];
    const int o = blockIdx.y;
    const int64_t r = blockIdx.x * (int64_t)kPairBlock + threadIdx.x;
    const int32_t v = r < n ? nbr[o * n + r] : -1;
    const unsigned bal = __ballot_sync(0xffffffffu, v >= 0);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (lane == 0) warp_cnt[w] = __popc(bal);
    __syncthreads();
    int before = 0;
    for (int k = 0; k < w; ++k) before += warp_cnt[k];
    if (v >= 0) {
        const int64_t pos = starts[o * nblk + blockIdx.x] + before + __popc(bal & ((1u << lane) - 1));
        pin[pos] = v;
        pout[pos] = (int32_t)r;
    }
}

// ---------------------------------------------------------------------------
// Scratch of s3dsp_kmap_pairs_noalloc: a file-scope device array, so the call
// allocates nothing. Layout: int32 counts[kNoAllocMaxBlocks] (one per offset
// and 1024-row block) | int64 starts[kNoAllocMaxBlocks + 1] (their exclusive
// prefix sums) | int64 offsets[32] (the kvol + 1 per-offset starts). Every
// element a call reads is written earlier in the same call, so nothing needs
// clearing between calls. Each device that loads the library holds this
// array (about 0.65 MiB) until the process exits.
// ---------------------------------------------------------------------------
constexpr int64_t kNoAllocMaxRows = 1ll << 21;  // 2,097,152 output rows
constexpr int64_t kNoAllocMaxBlocks = 27 * (kNoAllocMaxRows / kPairBlock);
constexpr size_t kNoAllocCountsBytes = (size_t)kNoAllocMaxBlocks * 4;
constexpr size_t kNoAllocStartsBytes = (size_t)(kNoAllocMaxBlocks + 1) * 8;
constexpr size_t kNoAllocBytes = kNoAllocCountsBytes + kNoAllocStartsBytes + 32 * 8;
static __device__ __align__(256) unsigned char g_pairs_scratch[kNoAllocBytes];

__global__ void pair_offsets_kernel(const int64_t* __restrict__ starts, int64_t nblk, int kvol, int64_t m,
                                    int64_t* __restrict__ offs) {
    pdl_wait();
    pdl_trigger();
    const int o = threadIdx.x;
    if (o < kvol) offs[o] = starts[o * nblk];
    if (o == kvol) offs[kvol] = starts[m];
}

// Device address of g_pairs_scratch on the current device. The host-side name
// of the array is only a stand-in, so the address comes from
// cudaGetSymbolAddress; it is looked up on every call (cheap after the first),
// so a module reloaded after cudaDeviceReset is never addressed through a
// stale pointer.
cudaError_t noalloc_scratch(unsigned char** out) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_pairs_scratch);
    if (e != cudaSuccess) return e;
    *out = static_cast<unsigned char*>(ptr);
    return cudaSuccess;
}

inline int grid_for(int64_t n, int threads, int sm_count) {
    int64_t g = (n + threads - 1) / threads;
    const int64_t cap = (int64_t)sm_count * 16;
    if (g > cap) g = cap;
    return (int)(g < 1 ? 1 : g);
}


// zero_mask: the builder ORs tile bits across blocks (a builder that stores
// every tile's mask whole passes false)
s3dsp_kmap* new_kmap(s3dsp_context* ctx, int64_t n_out, int64_t n_in, int kvol, bool zero_mask, cudaError_t* err) {
    auto* k = new (std::nothrow) s3dsp_kmap();
    if (!k) {
        *err = cudaErrorMemoryAllocation;
        return nullptr;
    }
    k->n_out = n_out;
    k->n_in = n_in;
    k->kvol = kvol;
    k->n_tiles = (n_out + kTileRows - 1) / kTileRows;
    *err = s3dsp::malloc_async(&k->nbr, sizeof(int32_t) * (size_t)kvol * (size_t)(n_out > 0 ? n_out : 1), ctx->stream);
    if (*err == cudaSuccess)
        *err = s3dsp::malloc_async(&k->tile_mask, sizeof(uint32_t) * (size_t)(k->n_tiles > 0 ? k->n_tiles : 1), ctx->stream);
    if (*err == cudaSuccess && zero_mask && k->n_tiles > 0)
        *err = cudaMemsetAsync(k->tile_mask, 0, sizeof(uint32_t) * (size_t)k->n_tiles, ctx->stream);
    if (*err != cudaSuccess) {
        if (k->nbr) cudaFreeAsync(k->nbr, ctx->stream);
        if (k->tile_mask) cudaFreeAsync(k->tile_mask, ctx->stream);
        delete k;
        return nullptr;
    }
    return k;
}

}  // namespace

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
extern "C" S3DSP_API s3d_status s3dsp_hash_build(s3dsp_context* ctx, const int32_t* d_coords,
                                                 int64_t n, int32_t reject_duplicates,
                                                 s3dsp_hash** out, char* error,
                                                 uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !out) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "ctx/out is NULL");
    *out = nullptr;
    if (n <= 0) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "coordinate count %lld <= 0", (long long)n);
    if (n > (1ll << 30)) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "coordinate count %lld > 2^30", (long long)n);
    if (!d_coords || ((uintptr_t)d_coords & 15))
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "d_coords must be a 16-byte aligned device pointer");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    auto* h = new (std::nothrow) s3dsp_hash();
    if (!h) return fail(error, error_capacity, S3D_OUT_OF_MEMORY, "hash allocation");
    h->n = n;
    h->reject_duplicates = reject_duplicates;
    // load factor <= 1/4: a warp waits for its longest probe sequence, and the
    // expected longest of 32 linear-probe sequences grows fast with the load
    uint64_t cap = 64;
    while (cap < 4 * (uint64_t)n) cap <<= 1;
    h->capacity = cap;
    cudaStream_t st = ctx->stream;
    // above 16 MB of table, probes mostly miss L2: map builders then read each
    // row's first row from a one-probe-per-row pass instead of probing again
    const bool self_pass = cap * 16 > (16ull << 20);
    cudaError_t e = s3dsp::malloc_async(&h->slots, cap * 16, st);
    if (e == cudaSuccess) e = s3dsp::malloc_async(&h->coords, (size_t)n * 16, st);
    if (e == cudaSuccess && self_pass) e = s3dsp::malloc_async(&h->self_row, (size_t)n * 4, st);
    if (e != cudaSuccess) {
        s3dsp_hash_free(ctx, h);
        return cuda_fail(error, error_capacity, e, "hash allocation");
    }
    const int threads = 256;
    e = launch_pdl(hash_init_kernel, dim3(grid_for((int64_t)cap, threads, ctx->sm_count)), dim3(threads), 0, st,
                   h->slots, cap);
    if (e == cudaSuccess)
        e = launch_pdl(hash_insert_kernel, dim3(grid_for(n, threads, ctx->sm_count)), dim3(threads), 0, st,
                       reinterpret_cast<const int4*>(d_coords), n, reinterpret_cast<int4*>(h->coords), h->slots,
                       (unsigned long long)(cap - 1), reject_duplicates, ctx->d_status);
    if (e == cudaSuccess && self_pass)
        e = launch_pdl(hash_self_kernel, dim3(grid_for(n, threads, ctx->sm_count)), dim3(threads), 0, st,
                       reinterpret_cast<const int4*>(h->coords), n, view_of(h), h->self_row);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) {
        s3dsp_hash_free(ctx, h);
        return cuda_fail(error, error_capacity, e, "hash kernels");
    }
    if (!(ctx->flags & S3DSP_CONTEXT_DEFERRED_CHECKS)) {
        const s3d_status s = check_status(ctx, error, error_capacity);
        if (s != S3D_OK) {
            s3dsp_hash_free(ctx, h);
            return s;
        }
    }
    *out = h;
    return S3D_OK;
}

extern "C" S3DSP_API void s3dsp_hash_free(s3dsp_context* ctx, s3dsp_hash* h) {
    if (!h) return;
    cudaStream_t st = ctx ? ctx->stream : nullptr;
    if (h->slots) cudaFreeAsync(h->slots, st);
    if (h->self_row) cudaFreeAsync(h->self_row, st);
    if (h->coords) cudaFreeAsync(h->coords, st);
    delete h;
}

extern "C" S3DSP_API int64_t s3dsp_hash_size(const s3dsp_hash* h) { return h ? h->n : 0; }

extern "C" S3DSP_API s3d_status s3dsp_hash_lookup(s3dsp_context* ctx, const s3dsp_hash* h,
                                                  const int32_t* d_query, int64_t m, int32_t* d_rows,
                                                  char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !h) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "ctx/hash is NULL");
    if (m < 0) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "negative query count");
    if (m == 0) return S3D_OK;
    if (!d_query || ((uintptr_t)d_query & 15) || !d_rows)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "query/rows pointers invalid");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    launch_pdl(hash_lookup_kernel, dim3(grid_for(m, 256, ctx->sm_count)), dim3(256), 0, ctx->stream,
               reinterpret_cast<const int4*>(d_query), m, view_of(h), d_rows);
    S3DSP_LAUNCH_CHECK("hash_lookup_kernel");
    return S3D_OK;
}

extern "C" S3DSP_API s3d_status s3dsp_kmap_build_subm3_range(s3dsp_context* ctx, const s3dsp_hash* h,
                                                             int64_t row_begin, int64_t row_end, s3dsp_kmap** out,
                                                             char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !h || !out) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    *out = nullptr;
    if (row_begin < 0 || row_end <= row_begin || row_end > h->n)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "rows [%lld, %lld) outside [0, %lld)",
                    (long long)row_begin, (long long)row_end, (long long)h->n);
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    cudaError_t e;
    const int64_t n_out = row_end - row_begin;
    s3dsp_kmap* k = new_kmap(ctx, n_out, h->n, 27, false, &e);
    if (!k) return cuda_fail(error, error_capacity, e, "kmap allocation");
    const int64_t tiles = (n_out + kTileRows - 1) / kTileRows;
    // output rows are hash rows row_begin ..; inputs are all its rows
    e = launch_pdl(kmap_subm3_kernel, dim3((unsigned)tiles), dim3(kTileRows * kSlabs), 0, ctx->stream,
                   reinterpret_cast<const int4*>(h->coords), row_begin, n_out, view_of(h),
                   static_cast<const int32_t*>(h->self_row), k->nbr, k->tile_mask);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) {
        s3dsp_kmap_free(ctx, k);
        return cuda_fail(error, error_capacity, e, "kmap_subm3_kernel");
    }
    *out = k;
    return S3D_OK;
}

extern "C" S3DSP_API s3d_status s3dsp_kmap_build_subm3_rows(s3dsp_context* ctx, const s3dsp_hash* h, int64_t n_out,
                                                            s3dsp_kmap** out, char* error, uint64_t error_capacity) {
    return s3dsp_kmap_build_subm3_range(ctx, h, 0, n_out, out, error, error_capacity);
}

extern "C" S3DSP_API s3d_status s3dsp_kmap_build_subm3(s3dsp_context* ctx, const s3dsp_hash* h,
                                                       s3dsp_kmap** out, char* error,
                                                       uint64_t error_capacity) {
    if (!h) {
        clear_error(error, error_capacity);
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    }
    return s3dsp_kmap_build_subm3_range(ctx, h, 0, h->n, out, error, error_capacity);
}

extern "C" S3DSP_API s3d_status s3dsp_subdivide(s3dsp_context* ctx, const s3dsp_hash* parents,
                                                int32_t* d_child_coords, s3dsp_kmap** out,
                                                char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !parents || !out || !d_child_coords)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    *out = nullptr;
    if (((uintptr_t)d_child_coords & 15))
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "d_child_coords must be 16-byte aligned");
    if (!parents->reject_duplicates)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT,
                    "subdivide needs a parent hash built with reject_duplicates");
    if (parents->n > INT32_MAX / 8)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "parent count exceeds INT32_MAX/8");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    cudaError_t e;
    const int64_t np = parents->n;
    s3dsp_kmap* k = new_kmap(ctx, np * 8, np * 8, 27, true, &e);
    if (!k) return cuda_fail(error, error_capacity, e, "kmap allocation");
    const int64_t blocks = (np + 31) / 32;
    launch_pdl(subdivide_kernel, dim3((unsigned)blocks), dim3(256), 0, ctx->stream,
               reinterpret_cast<const int4*>(parents->coords), np, view_of(parents),
               reinterpret_cast<int4*>(d_child_coords), k->nbr, k->tile_mask);
    e = cudaGetLastError();
    if (e != cudaSuccess) {
        s3dsp_kmap_free(ctx, k);
        return cuda_fail(error, error_capacity, e, "subdivide_kernel");
    }
    *out = k;
    return S3D_OK;
}

extern "C" S3DSP_API void s3dsp_kmap_free(s3dsp_context* ctx, s3dsp_kmap* k) {
    if (!k) return;
    cudaStream_t st = ctx ? ctx->stream : nullptr;
    if (k->nbr) cudaFreeAsync(k->nbr, st);
    if (k->tile_mask) cudaFreeAsync(k->tile_mask, st);
    delete k;
}

extern "C" S3DSP_API int64_t s3dsp_kmap_rows(const s3dsp_kmap* k) { return k ? k->n_out : 0; }

namespace {
// out[o][r] = rows[nbr[o][r]] (-1 stays -1); an entry of rows outside
// [0, n_rows_in) becomes -1 and sets kErrRowRange
__global__ void kmap_compose_kernel(const int32_t* __restrict__ nbr, int64_t total, const int32_t* __restrict__ rows,
                                    int64_t n_rows, int64_t n_rows_in, int32_t* __restrict__ out,
                                    uint32_t* __restrict__ status) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int32_t v = nbr[i];
        int32_t u = -1;
        if (v >= 0 && v < n_rows) {
            u = __ldg(rows + v);
            if (u < 0 || u >= n_rows_in) {
                atomicOr(status, kErrRowRange);
                u = -1;
            }
        }
        out[i] = u;
    }
}
}  // namespace

extern "C" S3DSP_API s3d_status s3dsp_kmap_compose(s3dsp_context* ctx, const s3dsp_kmap* k, const int32_t* d_rows,
                                                   int64_t n_rows_in, s3dsp_kmap** out, char* error,
                                                   uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !k || !d_rows || !out) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    *out = nullptr;
    if (n_rows_in < 0 || n_rows_in > INT32_MAX) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "bad n_rows_in");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    cudaError_t e;
    s3dsp_kmap* c = new_kmap(ctx, k->n_out, n_rows_in, k->kvol, false, &e);
    if (!c) return cuda_fail(error, error_capacity, e, "kmap allocation");
    const int64_t total = (int64_t)k->kvol * k->n_out;
    if (total > 0) {
        launch_pdl(kmap_compose_kernel, dim3(grid_for(total, 256, ctx->sm_count)), dim3(256), 0, ctx->stream, k->nbr,
                   total, d_rows, k->n_in, n_rows_in, c->nbr, ctx->d_status);
        e = cudaGetLastError();
        // the composed map has a neighbour exactly where the original has one
        if (e == cudaSuccess && k->n_tiles > 0)
            e = cudaMemcpyAsync(c->tile_mask, k->tile_mask, sizeof(uint32_t) * (size_t)k->n_tiles,
                                cudaMemcpyDeviceToDevice, ctx->stream);
        if (e != cudaSuccess) {
            s3dsp_kmap_free(ctx, c);
            return cuda_fail(error, error_capacity, e, "kmap_compose_kernel");
        }
    }
    *out = c;
    return S3D_OK;
}

extern "C" S3DSP_API s3d_status s3dsp_kmap_export_dense(s3dsp_context* ctx, const s3dsp_kmap* k,
                                                        uint32_t sentinel_mode, int32_t* d_out,
                                                        char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !k || !d_out) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    if (sentinel_mode != S3DSP_SENTINEL_SLAT_N && sentinel_mode != S3DSP_SENTINEL_MESH_NEG1)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "unknown sentinel mode %u", sentinel_mode);
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    const int32_t sentinel = sentinel_mode == S3DSP_SENTINEL_SLAT_N ? (int32_t)k->n_in : -1;
    launch_pdl(export_dense_kernel, dim3(grid_for(k->n_out * 27, 256, ctx->sm_count)), dim3(256), 0, ctx->stream,
               k->nbr, k->n_out, k->kvol, sentinel, d_out);
    S3DSP_LAUNCH_CHECK("export_dense_kernel");
    return S3D_OK;
}

extern "C" S3DSP_API s3d_status s3dsp_kmap_pairs(s3dsp_context* ctx, const s3dsp_kmap* k,
                                                 int32_t* d_in, int32_t* d_out, int64_t capacity,
                                                 int64_t* h_offsets, char* error,
                                                 uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !k || !d_in || !d_out || !h_offsets)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    const int64_t nblk = (k->n_out + kPairBlock - 1) / kPairBlock;
    const int64_t m = nblk * k->kvol;
    int32_t* counts = nullptr;
    int64_t* starts = nullptr;
    S3DSP_CUDA(s3dsp::malloc_async(&counts, sizeof(int32_t) * (size_t)(m > 0 ? m : 1), ctx->stream), "pairs scratch");
    cudaError_t e = s3dsp::malloc_async(&starts, sizeof(int64_t) * (size_t)(m + 1), ctx->stream);
    if (e != cudaSuccess) {
        cudaFreeAsync(counts, ctx->stream);
        return cuda_fail(error, error_capacity, e, "pairs scratch");
    }
    if (nblk > 0)
        launch_pdl(pair_count_kernel, dim3((unsigned)nblk, k->kvol), dim3(kPairBlock), 0, ctx->stream, k->nbr,
                   k->n_out, counts, nblk);
    launch_pdl(pair_scan_kernel, dim3(1), dim3(1024), 0, ctx->stream, counts, m, starts);
    // per-offset starts = starts[o * nblk]
    int64_t* host_starts = new int64_t[(size_t)m + 1];
    e = cudaMemcpyAsync(host_starts, starts, sizeof(int64_t) * (size_t)(m + 1), cudaMemcpyDeviceToHost, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    s3d_status st = S3D_OK;
    if (e != cudaSuccess) {
        st = cuda_fail(error, error_capacity, e, "pair counts");
    } else if (host_starts[m] > capacity) {
        st = fail(error, error_capacity, S3D_INVALID_ARGUMENT, "pair capacity %lld < %lld needed",
                  (long long)capacity, (long long)host_starts[m]);
    } else {
        for (int o = 0; o < k->kvol; ++o) h_offsets[o] = host_starts[o * nblk];
        h_offsets[k->kvol] = host_starts[m];
        if (nblk > 0)
            launch_pdl(pair_write_kernel, dim3((unsigned)nblk, k->kvol), dim3(kPairBlock), 0, ctx->stream,
                       k->nbr, k->n_out, starts, nblk, d_in, d_out);
        e = cudaGetLastError();
        if (e != cudaSuccess) st = cuda_fail(error, error_capacity, e, "pair_write_kernel");
    }
    delete[] host_starts;
    cudaFreeAsync(counts, ctx->stream);
    cudaFreeAsync(starts, ctx->stream);
    // synchronous: the pair lists are complete when the call returns
    e = cudaStreamSynchronize(ctx->stream);
    if (st == S3D_OK && e != cudaSuccess) st = cuda_fail(error, error_capacity, e, "cudaStreamSynchronize");
    return st;
}

extern "C" S3DSP_API s3d_status s3dsp_kmap_pairs_noalloc(s3dsp_context* ctx, const s3dsp_kmap* k, int32_t* d_in,
                                                         int32_t* d_out, int64_t capacity, int64_t* h_offsets,
                                                         char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !k || !d_in || !d_out || !h_offsets)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    if (k->n_out > kNoAllocMaxRows)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT,
                    "kernel map has %lld output rows; the allocation-free pair build is limited to %lld rows "
                    "(use s3dsp_kmap_pairs)",
                    (long long)k->n_out, (long long)kNoAllocMaxRows);
    // the scratch is laid out for at most 27 offsets (counts, starts, offs[32])
    if (k->kvol < 1 || k->kvol > 27)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT,
                    "kernel map has %d offsets; the allocation-free pair build supports at most 27", (int)k->kvol);
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    unsigned char* scratch = nullptr;
    S3DSP_CUDA(noalloc_scratch(&scratch), "cudaGetSymbolAddress(no-alloc scratch)");
    int32_t* counts = reinterpret_cast<int32_t*>(scratch);
    int64_t* starts = reinterpret_cast<int64_t*>(scratch + kNoAllocCountsBytes);
    int64_t* offs = reinterpret_cast<int64_t*>(scratch + kNoAllocCountsBytes + kNoAllocStartsBytes);
    const int64_t nblk = (k->n_out + kPairBlock - 1) / kPairBlock;
    const int64_t m = nblk * k->kvol;
    if (nblk > 0)
        launch_pdl(pair_count_kernel, dim3((unsigned)nblk, k->kvol), dim3(kPairBlock), 0, ctx->stream, k->nbr,
                   k->n_out, counts, nblk);
    launch_pdl(pair_scan_kernel, dim3(1), dim3(1024), 0, ctx->stream, counts, m, starts);
    launch_pdl(pair_offsets_kernel, dim3(1), dim3(32), 0, ctx->stream, starts, nblk, k->kvol, m, offs);
    S3DSP_LAUNCH_CHECK("pair count/scan kernels");
    S3DSP_CUDA(cudaMemcpyAsync(h_offsets, offs, sizeof(int64_t) * (size_t)(k->kvol + 1), cudaMemcpyDeviceToHost,
                               ctx->stream),
               "pair offsets readback");
    S3DSP_CUDA(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    if (h_offsets[k->kvol] > capacity)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "pair capacity %lld < %lld needed",
                    (long long)capacity, (long long)h_offsets[k->kvol]);
    if (nblk > 0)
        launch_pdl(pair_write_kernel, dim3((unsigned)nblk, k->kvol), dim3(kPairBlock), 0, ctx->stream, k->nbr,
                   k->n_out, starts, nblk, d_in, d_out);
    S3DSP_LAUNCH_CHECK("pair_write_kernel");
    // the write kernel reads the shared scratch: return only once it is done,
    // so that calls the host has ordered never overlap on the GPU
    S3DSP_CUDA(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    return S3D_OK;
}
