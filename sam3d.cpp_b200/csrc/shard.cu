// One large volume over several GPUs (one process per GPU): the Morton-slab
// plan and the one-voxel halo exchange.
//
// Plan (host, identical on every rank, no communication): the active voxels
// are sorted by 3D Morton code (x, y, z shifted to start at 0, 21 bits each,
// x-major interleave; batch 1 above bit 63) and cut into `world` contiguous
// ranges of n*r/world; rank r owns range r. Its own rows are ordered interior
// first (no 26-neighbour on another rank), then boundary, Morton order in
// each; its ghost rows are the other ranks' voxels with a 26-neighbour owned
// by r, grouped by owner and in Morton order within; its send list to rank p
// is its own rows with a 26-neighbour owned by p, in own-row order -- the same
// set and order as p's ghosts from r, so the rows land in place.
//
// Exchange: the send rows are gathered into one buffer, then one NCCL group of
// ncclSend / ncclRecv per peer moves them straight into the ghost rows
// [n_own, n_own + n_ghost). NCCL is bound at run time (an already loaded
// libnccl.so.2 -- e.g. the one a framework in the same process uses -- or the
// system one), so the library links no NCCL and every communicator passed in
// must come from that same NCCL instance (s3dsp_nccl_comm_create uses it).
//
// The reference runs one object on one device; there is no counterpart.
#include "s3dsp_internal.h"

#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <mutex>
#include <numeric>
#include <vector>

using namespace s3dsp;

struct s3dsp_shard {
    int32_t world = 1, rank = 0;
    std::vector<int64_t> own, ghost;         // global row ids
    std::vector<int64_t> recv_counts, send_counts;  // [world]
    std::vector<int64_t> send_rows;          // local own-row indices, grouped by destination
    int64_t n_interior = 0;
    int32_t* d_send = nullptr;  // device copy of send_rows (made by the first exchange)
    int device = -1;
};

namespace {

uint64_t spread21(uint64_t v) {
    v &= 0x1FFFFFull;
    v = (v | (v << 32)) & 0x1F00000000FFFFull;
    v = (v | (v << 16)) & 0x1F0000FF0000FFull;
    v = (v | (v << 8)) & 0x100F00F00F00F00Full;
    v = (v | (v << 4)) & 0x10C30C30C30C30C3ull;
    v = (v | (v << 2)) & 0x1249249249249249ull;
    return v;
}

// (b, x, y, z) -> one int64, order-preserving for |x|, |y|, |z| < 2^20
int64_t packed_key(int64_t b, int64_t x, int64_t y, int64_t z) {
    return (((b << 21) + (x + (1 << 20))) << 42) + ((y + (1 << 20)) << 21) + (z + (1 << 20));
}

// open-addressing map packed key -> lowest row holding it
struct KeyIndex {
    std::vector<int64_t> keys;
    std::vector<int64_t> rows;
    uint64_t mask = 0;
    static constexpr int64_t kEmpty = INT64_MIN;
    explicit KeyIndex(int64_t n) {
        uint64_t cap = 16;
        while (cap < (uint64_t)n * 2) cap <<= 1;
        keys.assign(cap, kEmpty);
        rows.assign(cap, -1);
        mask = cap - 1;
    }
    static uint64_t mix(uint64_t k) {
        k ^= k >> 33;
        k *= 0xff51afd7ed558ccdull;
        k ^= k >> 33;
        k *= 0xc4ceb9fe1a85ec53ull;
        k ^= k >> 33;
        return k;
    }
    void insert(int64_t key, int64_t row) {
        for (uint64_t s = mix((uint64_t)key) & mask;; s = (s + 1) & mask) {
            if (keys[s] == kEmpty) {
                keys[s] = key;
                rows[s] = row;
                return;
            }
            if (keys[s] == key) return;  // keep the lowest row (rows arrive in order)
        }
    }
    int64_t find(int64_t key) const {
        for (uint64_t s = mix((uint64_t)key) & mask;; s = (s + 1) & mask) {
            if (keys[s] == kEmpty) return -1;
            if (keys[s] == key) return rows[s];
        }
    }
};

// ---- NCCL, bound at run time -------------------------------------------------
struct NcclApi {
    bool ok = false;
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*group_start)() = nullptr;
    ncclResult_t (*group_end)() = nullptr;
    ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
};

const NcclApi& nccl_api() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h) return;
        auto sym = [&](const char* name) { return dlsym(h, name); };
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
        api.group_start = reinterpret_cast<decltype(api.group_start)>(sym("ncclGroupStart"));
        api.group_end = reinterpret_cast<decltype(api.group_end)>(sym("ncclGroupEnd"));
        api.send = reinterpret_cast<decltype(api.send)>(sym("ncclSend"));
        api.recv = reinterpret_cast<decltype(api.recv)>(sym("ncclRecv"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
        api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.group_start && api.group_end &&
                 api.send && api.recv && api.error_string;
    });
    return api;
}

__global__ void gather_rows_kernel(const uint8_t* __restrict__ x, const int32_t* __restrict__ rows, int64_t n_rows,
                                   int64_t row_bytes, uint8_t* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    // 16-byte words when rows allow it, else bytes
    if ((row_bytes & 15) == 0) {
        const int64_t words = row_bytes >> 4;
        const int64_t total = n_rows * words;
        for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
            const int64_t r = i / words, w = i - r * words;
            reinterpret_cast<uint4*>(out)[i] = reinterpret_cast<const uint4*>(x + (int64_t)rows[r] * row_bytes)[w];
        }
    } else {
        const int64_t total = n_rows * row_bytes;
        for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
            const int64_t r = i / row_bytes, b = i - r * row_bytes;
            out[i] = x[(int64_t)rows[r] * row_bytes + b];
        }
    }
}

}  // namespace

extern "C" {

S3DSP_API s3d_status s3dsp_shard_plan_morton(const int32_t* h_coords, int64_t n, int32_t world, int32_t rank,
                                             s3dsp_shard** out, char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!out || (n > 0 && !h_coords)) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    *out = nullptr;
    if (n < 0 || world < 1 || world > 32767 || rank < 0 || rank >= world)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "bad n / world / rank");
    // Morton codes
    int64_t mn[3] = {INT64_MAX, INT64_MAX, INT64_MAX}, mx[3] = {INT64_MIN, INT64_MIN, INT64_MIN};
    for (int64_t i = 0; i < n; ++i) {
        if (h_coords[4 * i] < 0 || h_coords[4 * i] > 1)
            return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "the Morton plan orders one object (batch 0 or 1)");
        for (int a = 0; a < 3; ++a) {
            mn[a] = std::min<int64_t>(mn[a], h_coords[4 * i + 1 + a]);
            mx[a] = std::max<int64_t>(mx[a], h_coords[4 * i + 1 + a]);
        }
    }
    for (int a = 0; a < 3 && n > 0; ++a)
        if (mx[a] - mn[a] >= (1 << 20))
            return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "coordinate extent exceeds 2^20 per axis");
    std::vector<uint64_t> code((size_t)n);
    for (int64_t i = 0; i < n; ++i) {
        const int32_t* c = h_coords + 4 * i;
        code[(size_t)i] = (spread21((uint64_t)(c[1] - mn[0])) << 2) | (spread21((uint64_t)(c[2] - mn[1])) << 1) |
                          spread21((uint64_t)(c[3] - mn[2])) | ((uint64_t)c[0] << 63);
    }
    std::vector<int64_t> order((size_t)n);
    std::iota(order.begin(), order.end(), 0);
    std::stable_sort(order.begin(), order.end(), [&](int64_t a, int64_t b) { return code[(size_t)a] < code[(size_t)b]; });
    std::vector<int64_t> pos((size_t)n), bounds((size_t)world + 1);
    for (int64_t i = 0; i < n; ++i) pos[(size_t)order[(size_t)i]] = i;
    for (int32_t r = 0; r <= world; ++r) bounds[(size_t)r] = n * r / world;
    std::vector<int32_t> owner((size_t)n);
    for (int32_t r = 0; r < world; ++r)
        for (int64_t i = bounds[(size_t)r]; i < bounds[(size_t)r + 1]; ++i) owner[(size_t)order[(size_t)i]] = r;
    // neighbour owners over the 26 offsets (dx, dy, dz lexicographic, centre skipped)
    KeyIndex idx(n);
    for (int64_t i = 0; i < n; ++i)
        idx.insert(packed_key(h_coords[4 * i], h_coords[4 * i + 1], h_coords[4 * i + 2], h_coords[4 * i + 3]), i);
    std::vector<int16_t> nb((size_t)n * 26);
    for (int64_t i = 0; i < n; ++i) {
        const int32_t* c = h_coords + 4 * i;
        int j = 0;
        for (int dx = -1; dx <= 1; ++dx)
            for (int dy = -1; dy <= 1; ++dy)
                for (int dz = -1; dz <= 1; ++dz) {
                    if (!dx && !dy && !dz) continue;
                    const int64_t v = idx.find(packed_key(c[0], (int64_t)c[1] + dx, (int64_t)c[2] + dy, (int64_t)c[3] + dz));
                    nb[(size_t)i * 26 + j++] = v < 0 ? (int16_t)-1 : (int16_t)owner[(size_t)v];
                }
    }
    auto touches = [&](int64_t v, int32_t r) {
        for (int j = 0; j < 26; ++j)
            if (nb[(size_t)v * 26 + j] == r) return true;
        return false;
    };
    auto* p = new (std::nothrow) s3dsp_shard;
    if (!p) return fail(error, error_capacity, S3D_OUT_OF_MEMORY, "host allocation");
    p->world = world;
    p->rank = rank;
    // own rows: interior first, then boundary, Morton order in each
    std::vector<int64_t> interior, boundary;
    for (int64_t i = bounds[(size_t)rank]; i < bounds[(size_t)rank + 1]; ++i) {
        const int64_t v = order[(size_t)i];
        bool b = false;
        for (int j = 0; j < 26 && !b; ++j) b = nb[(size_t)v * 26 + j] >= 0 && nb[(size_t)v * 26 + j] != rank;
        (b ? boundary : interior).push_back(v);
    }
    p->n_interior = (int64_t)interior.size();
    p->own = std::move(interior);
    p->own.insert(p->own.end(), boundary.begin(), boundary.end());
    // ghosts: other ranks' voxels touching rank, by (owner, Morton position)
    for (int64_t v = 0; v < n; ++v)
        if (owner[(size_t)v] != rank && touches(v, rank)) p->ghost.push_back(v);
    std::sort(p->ghost.begin(), p->ghost.end(), [&](int64_t a, int64_t b) {
        return owner[(size_t)a] != owner[(size_t)b] ? owner[(size_t)a] < owner[(size_t)b] : pos[(size_t)a] < pos[(size_t)b];
    });
    p->recv_counts.assign((size_t)world, 0);
    for (int64_t v : p->ghost) ++p->recv_counts[(size_t)owner[(size_t)v]];
    // sends: own rows touching each peer, in own-row order
    p->send_counts.assign((size_t)world, 0);
    for (int32_t q = 0; q < world; ++q) {
        if (q == rank) continue;
        for (size_t l = 0; l < p->own.size(); ++l)
            if (touches(p->own[l], q)) {
                p->send_rows.push_back((int64_t)l);
                ++p->send_counts[(size_t)q];
            }
    }
    *out = p;
    return S3D_OK;
}

S3DSP_API s3d_status s3dsp_shard_info(const s3dsp_shard* p, int64_t* n_own, int64_t* n_interior, int64_t* n_ghost,
                                      int64_t* n_send) {
    if (!p) return S3D_INVALID_ARGUMENT;
    if (n_own) *n_own = (int64_t)p->own.size();
    if (n_interior) *n_interior = p->n_interior;
    if (n_ghost) *n_ghost = (int64_t)p->ghost.size();
    if (n_send) *n_send = (int64_t)p->send_rows.size();
    return S3D_OK;
}

S3DSP_API s3d_status s3dsp_shard_lists(const s3dsp_shard* p, int64_t* h_own, int64_t* h_ghost, int64_t* h_recv_counts,
                                       int64_t* h_send_counts, int64_t* h_send_rows) {
    if (!p) return S3D_INVALID_ARGUMENT;
    auto put = [](int64_t* dst, const std::vector<int64_t>& v) {
        if (dst && !v.empty()) std::memcpy(dst, v.data(), v.size() * sizeof(int64_t));
    };
    put(h_own, p->own);
    put(h_ghost, p->ghost);
    put(h_recv_counts, p->recv_counts);
    put(h_send_counts, p->send_counts);
    put(h_send_rows, p->send_rows);
    return S3D_OK;
}

S3DSP_API void s3dsp_shard_free(s3dsp_context* ctx, s3dsp_shard* p) {
    if (!p) return;
    if (p->d_send) {
        if (ctx) cudaSetDevice(ctx->device);
        cudaFree(p->d_send);
    }
    delete p;
}

S3DSP_API s3d_status s3dsp_nccl_unique_id(uint8_t* id, char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    const NcclApi& api = nccl_api();
    if (!api.ok) return fail(error, error_capacity, S3D_INTERNAL_ERROR, "libnccl.so.2 could not be bound");
    if (!id) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    ncclUniqueId u;
    const ncclResult_t r = api.get_unique_id(&u);
    if (r != ncclSuccess) return fail(error, error_capacity, S3D_INTERNAL_ERROR, "ncclGetUniqueId: %s", api.error_string(r));
    std::memcpy(id, u.internal, sizeof u.internal);
    return S3D_OK;
}

S3DSP_API s3d_status s3dsp_nccl_comm_create(s3dsp_context* ctx, int32_t world, int32_t rank, const uint8_t* id,
                                            void** comm, char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    const NcclApi& api = nccl_api();
    if (!api.ok) return fail(error, error_capacity, S3D_INTERNAL_ERROR, "libnccl.so.2 could not be bound");
    if (!ctx || !id || !comm || world < 1 || rank < 0 || rank >= world)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "bad argument");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    ncclUniqueId u;
    std::memcpy(u.internal, id, sizeof u.internal);
    ncclComm_t c = nullptr;
    const ncclResult_t r = api.comm_init_rank(&c, world, u, rank);
    if (r != ncclSuccess) return fail(error, error_capacity, S3D_INTERNAL_ERROR, "ncclCommInitRank: %s", api.error_string(r));
    *comm = c;
    return S3D_OK;
}

S3DSP_API void s3dsp_nccl_comm_free(void* comm) {
    const NcclApi& api = nccl_api();
    if (comm && api.ok) api.comm_destroy(static_cast<ncclComm_t>(comm));
}

S3DSP_API s3d_status s3dsp_halo_exchange(s3dsp_context* ctx, s3dsp_shard* p, void* comm, void* d_x, int64_t c,
                                         uint32_t dtype, char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !p || !d_x || c <= 0 || !dtype_ok(dtype))
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "bad argument");
    if (p->world == 1) return S3D_OK;
    if (!comm) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL communicator");
    const NcclApi& api = nccl_api();
    if (!api.ok) return fail(error, error_capacity, S3D_INTERNAL_ERROR, "libnccl.so.2 could not be bound");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    cudaStream_t st = ctx->stream;
    const int64_t n_send = (int64_t)p->send_rows.size();
    if (n_send > 0 && (!p->d_send || p->device != ctx->device)) {  // send rows copied to the device once
        if (p->d_send) cudaFree(p->d_send);
        p->d_send = nullptr;
        std::vector<int32_t> rows(p->send_rows.begin(), p->send_rows.end());
        S3DSP_CUDA(cudaMalloc(&p->d_send, 4 * (size_t)n_send), "send rows");
        S3DSP_CUDA(cudaMemcpy(p->d_send, rows.data(), 4 * (size_t)n_send, cudaMemcpyHostToDevice), "send rows");
        p->device = ctx->device;
    }
    const int64_t row_bytes = c * (int64_t)dtype_size(dtype);
    uint8_t* x = static_cast<uint8_t*>(d_x);
    uint8_t* send = nullptr;
    if (n_send > 0) {
        S3DSP_CUDA(s3dsp::malloc_async(&send, (size_t)(n_send * row_bytes), st), "send buffer");
        const int64_t work = (row_bytes & 15) == 0 ? n_send * (row_bytes >> 4) : n_send * row_bytes;
        int64_t g = (work + 255) / 256;
        if (g > ctx->sm_count * 8) g = ctx->sm_count * 8;
        launch_pdl(gather_rows_kernel, dim3((int)(g < 1 ? 1 : g)), dim3(256), 0, st, x, p->d_send, n_send, row_bytes,
                   send);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) {
            cudaFreeAsync(send, st);
            return cuda_fail(error, error_capacity, e, "gather_rows_kernel");
        }
    }
    ncclComm_t cm = static_cast<ncclComm_t>(comm);
    ncclResult_t r = api.group_start();
    int64_t so = 0, ro = (int64_t)p->own.size();
    for (int32_t q = 0; q < p->world && r == ncclSuccess; ++q) {
        const int64_t ns = p->send_counts[(size_t)q], nr = p->recv_counts[(size_t)q];
        if (ns > 0) r = api.send(send + so * row_bytes, (size_t)(ns * row_bytes), ncclUint8, q, cm, st);
        if (r == ncclSuccess && nr > 0) r = api.recv(x + ro * row_bytes, (size_t)(nr * row_bytes), ncclUint8, q, cm, st);
        so += ns;
        ro += nr;
    }
    const ncclResult_t r2 = api.group_end();
    if (send) cudaFreeAsync(send, st);
    if (r != ncclSuccess || r2 != ncclSuccess)
        return fail(error, error_capacity, S3D_INTERNAL_ERROR, "NCCL halo exchange: %s",
                    api.error_string(r != ncclSuccess ? r : r2));
    return S3D_OK;
}

}  // extern "C"
