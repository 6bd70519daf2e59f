// Internal declarations shared by the s3dsp translation units.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <new>
#include <utility>

#include "s3dsp.h"

// ---------------------------------------------------------------------------
// device status words (written by kernels that validate their inputs)
// ---------------------------------------------------------------------------
enum : uint32_t {
    kErrCoordRange = 1u << 0,   // coordinate outside the packed key domain
    kErrHashFull = 1u << 1,     // probe bound exceeded (never with load <= 1/2)
    kErrDuplicate = 1u << 2,    // duplicate coordinate where duplicates are rejected
    kErrPipelineTimeout = 1u << 3,  // a bounded device wait gave up
    kErrRowRange = 1u << 4,     // a caller-supplied row index outside its table (read as "no row")
};

// S3DSP_CONTEXT_COPY_STREAMS: the host-buffer pipeline of a context. Call j
// of the queued host-buffer entry points uses staging slot j % kSlots: its
// host -> device copies run on copy_in, its kernels on the context's stream,
// its device -> host copy on copy_out, ordered by the slot's events. A slot
// is reused three calls later, once its previous inputs are consumed
// (comp_done) and its previous output copied out (out_done).
struct s3dsp_host_pipe {
    static constexpr int kSlots = 3;
    struct Slot {
        void* d_coords = nullptr;
        void* d_x = nullptr;
        void* d_out = nullptr;
        size_t coords_bytes = 0, x_bytes = 0, out_bytes = 0;
        cudaEvent_t in_done = nullptr, comp_done = nullptr, out_done = nullptr;
        bool used = false;
    };
    cudaStream_t copy_in = nullptr, copy_out = nullptr;
    cudaEvent_t order = nullptr;  // fork / join
    Slot slots[kSlots];
    uint64_t calls = 0;
};

struct s3dsp_context {
    int device = 0;
    cudaStream_t stream = nullptr;
    bool owns_stream = false;
    uint32_t flags = 0;
    int sm_count = 0;      // SMs the context's grids are sized for (s3dsp_context_set_sm_limit)
    int sm_device = 0;     // SMs of the device
    uint32_t* d_status = nullptr;  // [4] error bits, duplicate count, ...
    s3dsp_host_pipe* pipe = nullptr;  // S3DSP_CONTEXT_COPY_STREAMS only
};

struct s3dsp_hash {
    int64_t n = 0;
    uint64_t capacity = 0;               // power of two >= 4n
    ulonglong2* slots = nullptr;         // [capacity] {packed key, first row in the low 32 bits}
    int32_t* coords = nullptr;           // [n, 4] own copy
    int32_t* self_row = nullptr;         // [n] first row holding each row's key, or null (small tables)
    int32_t reject_duplicates = 0;
};

struct s3dsp_kmap {
    int64_t n_out = 0;
    int64_t n_in = 0;
    int32_t kvol = 27;
    int32_t* nbr = nullptr;         // [kvol][n_out], -1 = none
    uint32_t* tile_mask = nullptr;  // [ceil(n_out / 128)] bit o = any neighbour at offset o
    int64_t n_tiles = 0;
};

namespace s3dsp {

constexpr int kTileRows = 128;  // rows per conv tile (tcgen05 M) == tile_mask granularity
constexpr int kSmemOptIn = 232448;  // opt-in dynamic shared memory per block (227 KB)

// Opt a kernel in to the full dynamic shared memory once per device (device
// < 64); later calls, including ones made during a stream capture, skip the
// attribute call.
inline cudaError_t smem_optin(const void* fn, int device, std::atomic<uint64_t>& done) {
    const uint64_t bit = 1ull << (device & 63);
    if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemOptIn);
    if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_acq_rel);
    return e;
}

// Programmatic dependent launch. A kernel launched by launch_pdl may start
// while the kernel before it on the stream is still finishing; it calls
// pdl_wait() before its first global-memory access (read or write), which
// returns once that kernel has completed and its writes are visible, and then
// pdl_trigger() so that the next launch_pdl kernel may be scheduled. Work
// before pdl_wait() touches shared memory, TMEM and kernel parameters only.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// (d0, d1) = (a * b0 + d0, a * b1 + d1), one packed two-lane FP32 FMA: each
// lane rounds once, like fmaf, so a loop of them gives the same bits as the
// scalar loop with half the FMA instructions (sm_100: fma.rn.f32x2)
__device__ __forceinline__ void fma2(float& d0, float& d1, float a, float b0, float b1) {
    asm("{\n\t.reg .b64 d, x, y;\n\t"
        "mov.b64 d, {%0, %1};\n\t"
        "mov.b64 x, {%2, %2};\n\t"
        "mov.b64 y, {%3, %4};\n\t"
        "fma.rn.f32x2 d, x, y, d;\n\t"
        "mov.b64 {%0, %1}, d;\n\t}"
        : "+f"(d0), "+f"(d1)
        : "f"(a), "f"(b0), "f"(b1));
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// error-buffer helpers (reference convention: include/sam3d.h:32-34)
inline void clear_error(char* error, uint64_t cap) {
    if (error && cap) error[0] = '\0';
}
inline s3d_status fail(char* error, uint64_t cap, s3d_status st, const char* fmt, ...) {
    if (error && cap) {
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(error, (size_t)cap, fmt, ap);
        va_end(ap);
        error[cap - 1] = '\0';
    }
    return st;
}
inline s3d_status cuda_fail(char* error, uint64_t cap, cudaError_t e, const char* what) {
    return fail(error, cap, e == cudaErrorMemoryAllocation ? S3D_OUT_OF_MEMORY : S3D_INTERNAL_ERROR,
                "%s: %s", what, cudaGetErrorString(e));
}

#define S3DSP_CUDA(call, what)                                              \
    do {                                                                    \
        cudaError_t e_ = (call);                                            \
        if (e_ != cudaSuccess) return ::s3dsp::cuda_fail(error, error_capacity, e_, what); \
    } while (0)

#define S3DSP_LAUNCH_CHECK(what)                                            \
    do {                                                                    \
        cudaError_t e_ = cudaGetLastError();                                \
        if (e_ != cudaSuccess) return ::s3dsp::cuda_fail(error, error_capacity, e_, what); \
    } while (0)

// The library's own stream-ordered memory pool on `device` (< 64), created on
// first use with an unlimited release threshold: hash tables, kernel maps and
// scratch are rebuilt per object, and returning pool memory to the driver at
// every synchronisation would cost milliseconds of re-mapping. A private pool
// leaves the allocator policy of the host process (the device's default pool)
// untouched. s3dsp_context_create makes it, so no later call (inside a stream
// capture, say) has to.
cudaError_t lib_pool(int device, cudaMemPool_t* out);

// cudaMallocAsync from the library pool of the current device.
template <typename T>
inline cudaError_t malloc_async(T** p, size_t bytes, cudaStream_t stream) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    cudaMemPool_t pool;
    e = lib_pool(dev, &pool);
    if (e != cudaSuccess) return e;
    return cudaMallocFromPoolAsync(reinterpret_cast<void**>(p), bytes, pool, stream);
}

inline size_t dtype_size(uint32_t dt) { return dt == S3DSP_F32 ? 4 : 2; }
inline bool dtype_ok(uint32_t dt) { return dt == S3DSP_F32 || dt == S3DSP_BF16 || dt == S3DSP_F16; }

// Reads back the device status words and turns them into a status.
// return a C-ABI call's status when it is not S3D_OK
#define S3DSP_TRY(call)               \
    do {                              \
        const s3d_status s_ = (call); \
        if (s_ != S3D_OK) return s_;  \
    } while (0)

s3d_status check_status(s3dsp_context* ctx, char* error, uint64_t error_capacity);

// Orders the context's stream after everything queued so far on its copy
// streams (no-op without S3DSP_CONTEXT_COPY_STREAMS).
cudaError_t pipe_join(s3dsp_context* ctx);

// launch helpers implemented in the .cu files
//
// Every conv gathers its input rows from one or two sources: channels
// [0, cin_a) of a row come from `in` (row stride cin_a), channels [cin_a, cin)
// from `in_b` (row stride cin - cin_a), the same row index in both -- the
// channel concat of two tensors (ggml_concat(a, b, 0)) without building it.
// One source: in_b == nullptr, cin_a == cin.
cudaError_t launch_conv_f32(s3dsp_context* ctx, const s3dsp_kmap* kmap, int kvol, const float* in,
                            const float* in_b, int cin_a, int64_t n_in, int cin, int in_shift, const float* w,
                            const float* bias, const void* residual, uint32_t res_dtype,
                            int res_shift, void* out, uint32_t out_dtype, int64_t n_out, int cout,
                            uint32_t flags, const float* pro_sub, const float* pro_mul,
                            const float* pro_add, double* gn_partials, int gn_groups);
cudaError_t launch_conv_tc(s3dsp_context* ctx, const s3dsp_kmap* kmap, int kvol,
                           const __nv_bfloat16* in, const __nv_bfloat16* in_b, int cin_a, int64_t n_in, int cin,
                           int in_shift, const __nv_bfloat16* w, const float* bias, const void* residual,
                           uint32_t res_dtype, int res_shift, void* out, uint32_t out_dtype,
                           int64_t n_out, int cout, uint32_t flags, double* gn_partials,
                           int gn_groups, char* error, uint64_t error_capacity, s3d_status* st);
// 3xTF32 on the 128-row tensor-core kernel: in_hi / in_lo (and in_hi_b /
// in_lo_b for a second source) are the input split by s3dsp::split_tf32, w a
// weight packed for S3DSP_PREC_F32_3XTF32
cudaError_t launch_conv_tf32x3(s3dsp_context* ctx, const s3dsp_kmap* kmap, int kvol, const float* in_hi,
                               const float* in_lo, const float* in_hi_b, const float* in_lo_b, int cin_a, int cin,
                               int in_shift, const float* w, const float* bias,
                               const void* residual, uint32_t res_dtype, int res_shift, void* out, uint32_t out_dtype,
                               int64_t n_out, int cout, uint32_t flags, double* gn_partials, int gn_groups,
                               char* error, uint64_t error_capacity, s3d_status* st);
// x -> (TF32 high part, f32 remainder), n elements, on ctx's stream
cudaError_t split_tf32(s3dsp_context* ctx, const float* x, int64_t n, float* hi, float* lo);
// output columns per tensor-core tile for a layer of `cout` channels
int tc_pick_bn(int cout);
// rows: 128 or 256 output rows per stream-K work tile; csplit 2: one CTA pair
// (a cluster of 2) per 256-row work tile, the kernel offsets split between them
cudaError_t launch_conv_sk(s3dsp_context* ctx, const s3dsp_kmap* kmap, int kvol,
                           const __nv_bfloat16* in, const __nv_bfloat16* in_b, int cin_a, int64_t n_in, int cin,
                           int in_shift, const __nv_bfloat16* w, const float* bias, const void* residual,
                           uint32_t res_dtype, int res_shift, void* out, uint32_t out_dtype,
                           int64_t n_out, int cout, uint32_t flags, double* gn_partials,
                           int gn_groups, int rows, int csplit, char* error, uint64_t error_capacity,
                           s3d_status* st);
// per-tile input halos (one source, cin <= 256, cout <= 128): the plan for a
// layer (false: the kernel does not take it), and the launch
bool conv_halo_plan(int cin, int cout, int kvol, int in_shift, int* stages, int* halo_cap, int* per_sm);
cudaError_t launch_conv_halo(s3dsp_context* ctx, const s3dsp_kmap* kmap, int kvol, const __nv_bfloat16* in, int cin,
                             int in_shift, const __nv_bfloat16* w, const float* bias, const void* residual,
                             uint32_t res_dtype, int res_shift, void* out, uint32_t out_dtype, int64_t n_out, int cout,
                             uint32_t flags, double* gn_partials, int gn_groups, char* error, uint64_t error_capacity,
                             s3d_status* st);

}  // namespace s3dsp
