// Block-level host drivers: the host C++ that replaces the reference's GGML
// graph for one sparse block, composed from the library's kernels.
//   s3dsp_res_block_gn        conv3 -> GroupNorm -> SiLU -> conv3 -> + x
//                             (the config-2 benchmark block; GroupNorm as in
//                             mesh_decoder_graph.cpp:16-30)
//   s3dsp_mesh_upsample_level MeshUpsampleGraph::build, mesh_decoder_graph.cpp:42-132
//   s3dsp_slat_res_block      res_block of slat_flow_graph.cpp:216-275
// Scratch comes from the device's stream-ordered pool on the context stream.
#include "s3dsp_internal.h"

using namespace s3dsp;

namespace {

// RAII list of stream-ordered scratch allocations
struct Scratch {
    cudaStream_t st;
    void* ptrs[16] = {};
    int n = 0;
    explicit Scratch(cudaStream_t s) : st(s) {}
    ~Scratch() {
        for (int i = 0; i < n; ++i)
            if (ptrs[i]) cudaFreeAsync(ptrs[i], st);
    }
    template <class T>
    cudaError_t get(T** p, size_t bytes) {
        void* q = nullptr;
        const cudaError_t e = s3dsp::malloc_async(&q, bytes > 0 ? bytes : 16, st);
        if (e != cudaSuccess) return e;
        ptrs[n++] = q;
        *p = static_cast<T*>(q);
        return cudaSuccess;
    }
};

}  // namespace

extern "C" S3DSP_API s3d_status s3dsp_res_block_gn(s3dsp_context* ctx, const s3dsp_kmap* kmap, uint32_t precision,
                                                   const float* x, int64_t n, int64_t c, const void* w1,
                                                   const float* b1, const float* gamma, const float* beta,
                                                   const void* w2, const float* b2, int32_t groups, float eps,
                                                   float* out, char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !kmap || !x || !w1 || !w2 || !out) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    if (n != kmap->n_out) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "n != kmap rows");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    Scratch sc(ctx->stream);
    double* part;
    float *sub, *mul, *add, *y1;
    S3DSP_CUDA(sc.get(&part, sizeof(double) * (size_t)s3dsp_gn_partials_count(n, c, groups)), "scratch");
    S3DSP_CUDA(sc.get(&sub, 4 * (size_t)c), "scratch");
    S3DSP_CUDA(sc.get(&mul, 4 * (size_t)c), "scratch");
    S3DSP_CUDA(sc.get(&add, 4 * (size_t)c), "scratch");
    S3DSP_CUDA(sc.get(&y1, 4 * (size_t)(n * c)), "scratch");
    if (precision == S3DSP_PREC_F32_STRICT) {
        S3DSP_TRY(s3dsp_conv(ctx, kmap, 27, precision, x, S3DSP_F32, n, c, 0, w1, b1, nullptr, 0, 0, y1, S3DSP_F32, n, c,
                             0, nullptr, nullptr, nullptr, part, groups, error, error_capacity));
        S3DSP_TRY(s3dsp_gn_finalize(ctx, part, n, c, groups, eps, gamma, beta, sub, mul, add, error, error_capacity));
        return s3dsp_conv(ctx, kmap, 27, precision, y1, S3DSP_F32, n, c, 0, w2, b2, x, S3DSP_F32, 0, out, S3DSP_F32, n,
                          c, S3DSP_PRO_AFFINE_SILU, sub, mul, add, nullptr, 0, error, error_capacity);
    }
    // tensor-core precisions read their activations materialised: bf16 for BF16,
    // f32 for 3xTF32 (GN + SiLU applied by s3dsp_channel_affine, not a prologue)
    // BF16: conv1's output is stored in bf16 (its GroupNorm partial sums come
    // from the f32 accumulators before rounding) and GN + SiLU read it back
    // in bf16, halving that round trip
    const bool bf = precision == S3DSP_PREC_BF16;
    const uint32_t adt = bf ? S3DSP_BF16 : S3DSP_F32;
    const void* xin = x;
    void* hb;
    if (bf) {
        __nv_bfloat16* xb;
        S3DSP_CUDA(sc.get(&xb, 2 * (size_t)(n * c)), "scratch");
        S3DSP_TRY(s3dsp_convert(ctx, x, S3DSP_F32, xb, S3DSP_BF16, n * c, error, error_capacity));
        xin = xb;
    }
    S3DSP_CUDA(sc.get(&hb, dtype_size(adt) * (size_t)(n * c)), "scratch");
    S3DSP_TRY(s3dsp_conv(ctx, kmap, 27, precision, xin, adt, n, c, 0, w1, b1, nullptr, 0, 0, y1, adt, n, c, 0,
                         nullptr, nullptr, nullptr, part, groups, error, error_capacity));
    S3DSP_TRY(s3dsp_gn_finalize(ctx, part, n, c, groups, eps, gamma, beta, sub, mul, add, error, error_capacity));
    S3DSP_TRY(s3dsp_channel_affine(ctx, y1, adt, n, c, sub, mul, add, 1, hb, adt, error, error_capacity));
    return s3dsp_conv(ctx, kmap, 27, precision, hb, adt, n, c, 0, w2, b2, x, S3DSP_F32, 0, out, S3DSP_F32, n, c, 0,
                      nullptr, nullptr, nullptr, nullptr, 0, error, error_capacity);
}

extern "C" S3DSP_API s3d_status s3dsp_mesh_upsample_level(
    s3dsp_context* ctx, const s3dsp_hash* parents, uint32_t precision, const float* x, int64_t cin, int64_t cout,
    const float* gn1_w, const float* gn1_b, const void* conv1_w, const float* conv1_b, const float* gn2_w,
    const float* gn2_b, const void* conv2_w, const float* conv2_b, const void* skip_w, const float* skip_b,
    int32_t* child_coords, float* out, char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !parents || !x || !conv1_w || !conv2_w || !skip_w || !child_coords || !out)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    const int64_t np = parents->n, nc = 8 * np;
    const int groups = 32;
    const float eps = 1e-5f;  // SparseGroupNorm32 (mesh_decoder_graph.cpp:23)
    s3dsp_kmap* kmap = nullptr;
    S3DSP_TRY(s3dsp_subdivide(ctx, parents, child_coords, &kmap, error, error_capacity));
    struct KmapGuard {
        s3dsp_context* c;
        s3dsp_kmap* k;
        ~KmapGuard() { s3dsp_kmap_free(c, k); }
    } guard{ctx, kmap};
    Scratch sc(ctx->stream);
    const int64_t gmax = np > nc ? np : nc;
    double* part;
    float *sub1, *mul1, *add1, *sub2, *mul2, *add2, *y1, *skip;
    S3DSP_CUDA(sc.get(&part, sizeof(double) * (size_t)s3dsp_gn_partials_count(gmax, 1, groups)), "scratch");
    S3DSP_CUDA(sc.get(&sub1, 4 * (size_t)cin), "scratch");
    S3DSP_CUDA(sc.get(&mul1, 4 * (size_t)cin), "scratch");
    S3DSP_CUDA(sc.get(&add1, 4 * (size_t)cin), "scratch");
    S3DSP_CUDA(sc.get(&sub2, 4 * (size_t)cout), "scratch");
    S3DSP_CUDA(sc.get(&mul2, 4 * (size_t)cout), "scratch");
    S3DSP_CUDA(sc.get(&add2, 4 * (size_t)cout), "scratch");
    S3DSP_CUDA(sc.get(&y1, 4 * (size_t)(nc * cout)), "scratch");
    S3DSP_CUDA(sc.get(&skip, 4 * (size_t)(np * cout)), "scratch");
    // norm1 + silu1 on the parents (subdivide copies them to the 8 children)
    S3DSP_TRY(s3dsp_gn_stats(ctx, x, S3DSP_F32, np, cin, groups, part, error, error_capacity));
    S3DSP_TRY(s3dsp_gn_finalize(ctx, part, np, cin, groups, eps, gn1_w, gn1_b, sub1, mul1, add1, error, error_capacity));
    if (precision == S3DSP_PREC_F32_STRICT) {
        // conv1 over the children, gathering parent rows, GN1+SiLU in its prologue
        S3DSP_TRY(s3dsp_conv(ctx, kmap, 27, precision, x, S3DSP_F32, np, cin, 3, conv1_w, conv1_b, nullptr, 0, 0, y1,
                             S3DSP_F32, nc, cout, S3DSP_PRO_AFFINE_SILU, sub1, mul1, add1, part, groups, error,
                             error_capacity));
        S3DSP_TRY(s3dsp_gn_finalize(ctx, part, nc, cout, groups, eps, gn2_w, gn2_b, sub2, mul2, add2, error, error_capacity));
        // skip: 1x1 conv on the parents (== on the repeated input), broadcast to children
        S3DSP_TRY(s3dsp_conv(ctx, nullptr, 1, precision, x, S3DSP_F32, np, cin, 0, skip_w, skip_b, nullptr, 0, 0, skip,
                             S3DSP_F32, np, cout, 0, nullptr, nullptr, nullptr, nullptr, 0, error, error_capacity));
        return s3dsp_conv(ctx, kmap, 27, precision, y1, S3DSP_F32, nc, cout, 0, conv2_w, conv2_b, skip, S3DSP_F32, 3,
                          out, S3DSP_F32, nc, cout, S3DSP_PRO_AFFINE_SILU, sub2, mul2, add2, nullptr, 0, error,
                          error_capacity);
    }
    // tensor-core precisions: activations materialised as bf16 (BF16) or f32 (3xTF32)
    const bool bf = precision == S3DSP_PREC_BF16;
    const uint32_t adt = bf ? S3DSP_BF16 : S3DSP_F32;
    const size_t asz = dtype_size(adt);
    void *h1, *h2;
    const void* xin = x;
    S3DSP_CUDA(sc.get(&h1, asz * (size_t)(np * cin)), "scratch");
    S3DSP_CUDA(sc.get(&h2, asz * (size_t)(nc * cout)), "scratch");
    if (bf) {
        __nv_bfloat16* xb;
        S3DSP_CUDA(sc.get(&xb, 2 * (size_t)(np * cin)), "scratch");
        S3DSP_TRY(s3dsp_convert(ctx, x, S3DSP_F32, xb, S3DSP_BF16, np * cin, error, error_capacity));
        xin = xb;
    }
    S3DSP_TRY(s3dsp_channel_affine(ctx, x, S3DSP_F32, np, cin, sub1, mul1, add1, 1, h1, adt, error, error_capacity));
    // conv1's output in the activation dtype (bf16 for BF16: GN2 partials come
    // from the f32 accumulators, the bf16 copy is only what GN2 + SiLU read)
    S3DSP_TRY(s3dsp_conv(ctx, kmap, 27, precision, h1, adt, np, cin, 3, conv1_w, conv1_b, nullptr, 0, 0, y1, adt,
                         nc, cout, 0, nullptr, nullptr, nullptr, part, groups, error, error_capacity));
    S3DSP_TRY(s3dsp_gn_finalize(ctx, part, nc, cout, groups, eps, gn2_w, gn2_b, sub2, mul2, add2, error, error_capacity));
    S3DSP_TRY(s3dsp_channel_affine(ctx, y1, adt, nc, cout, sub2, mul2, add2, 1, h2, adt, error, error_capacity));
    S3DSP_TRY(s3dsp_conv(ctx, nullptr, 1, precision, xin, adt, np, cin, 0, skip_w, skip_b, nullptr, 0, 0, skip,
                         S3DSP_F32, np, cout, 0, nullptr, nullptr, nullptr, nullptr, 0, error, error_capacity));
    return s3dsp_conv(ctx, kmap, 27, precision, h2, adt, nc, cout, 0, conv2_w, conv2_b, skip, S3DSP_F32, 3, out,
                      S3DSP_F32, nc, cout, 0, nullptr, nullptr, nullptr, nullptr, 0, error, error_capacity);
}

extern "C" S3DSP_API s3d_status s3dsp_slat_res_block(s3dsp_context* ctx, const s3dsp_kmap* kmap, uint32_t precision,
                                                     const float* x, int64_t n, int64_t cin, int64_t cout,
                                                     const float* norm1_w, const float* norm1_b, const void* conv1_w,
                                                     const float* conv1_b, const float* mod_scale,
                                                     const float* mod_shift, const void* conv2_w, const float* conv2_b,
                                                     const void* skip_w, const float* skip_b, float* out, char* error,
                                                     uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !kmap || !x || !conv1_w || !conv2_w || !out)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    if (n != kmap->n_out) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "n != kmap rows");
    if (cin != cout && !skip_w)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "cin != cout needs a skip Linear (slat_flow_graph.cpp:266-272)");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    const float eps = 1e-6f;  // gb_layer_norm in res_block (slat_flow_graph.cpp:245-255)
    const bool bf = precision == S3DSP_PREC_BF16;
    const uint32_t hdt = bf ? S3DSP_BF16 : S3DSP_F32;
    const size_t hsz = bf ? 2 : 4;
    Scratch sc(ctx->stream);
    void *h1, *h2;
    float *y1, *skip = nullptr;
    S3DSP_CUDA(sc.get(&h1, hsz * (size_t)(n * cin)), "scratch");
    S3DSP_CUDA(sc.get(&h2, hsz * (size_t)(n * cout)), "scratch");
    S3DSP_CUDA(sc.get(&y1, 4 * (size_t)(n * cout)), "scratch");
    // norm1 (affine) -> SiLU -> conv1
    S3DSP_TRY(s3dsp_layer_norm(ctx, x, S3DSP_F32, n, cin, eps, norm1_w, norm1_b, nullptr, nullptr, 1, h1, hdt, error,
                               error_capacity));
    S3DSP_TRY(s3dsp_conv(ctx, kmap, 27, precision, h1, hdt, n, cin, 0, conv1_w, conv1_b, nullptr, 0, 0, y1, S3DSP_F32,
                         n, cout, 0, nullptr, nullptr, nullptr, nullptr, 0, error, error_capacity));
    // norm2 (no affine) -> modulate -> SiLU
    S3DSP_TRY(s3dsp_layer_norm(ctx, y1, S3DSP_F32, n, cout, eps, nullptr, nullptr, mod_scale, mod_shift, 1, h2, hdt,
                               error, error_capacity));
    // skip: identity, or Linear when the width changes
    const float* res = x;
    if (cin != cout) {
        S3DSP_CUDA(sc.get(&skip, 4 * (size_t)(n * cout)), "scratch");
        const void* xin = x;
        if (bf) {
            __nv_bfloat16* xb;
            S3DSP_CUDA(sc.get(&xb, 2 * (size_t)(n * cin)), "scratch");
            S3DSP_TRY(s3dsp_convert(ctx, x, S3DSP_F32, xb, S3DSP_BF16, n * cin, error, error_capacity));
            xin = xb;
        }
        S3DSP_TRY(s3dsp_conv(ctx, nullptr, 1, precision, xin, hdt, n, cin, 0, skip_w, skip_b, nullptr, 0, 0, skip,
                             S3DSP_F32, n, cout, 0, nullptr, nullptr, nullptr, nullptr, 0, error, error_capacity));
        res = skip;
    }
    return s3dsp_conv(ctx, kmap, 27, precision, h2, hdt, n, cout, 0, conv2_w, conv2_b, res, S3DSP_F32, 0, out, S3DSP_F32,
                      n, cout, 0, nullptr, nullptr, nullptr, nullptr, 0, error, error_capacity);
}

namespace {
// y[r] = x[rows[r]] for f32 rows of c channels (c % 4 == 0, 16-byte rows); a
// row index outside [0, n_in) gives a zero row and sets kErrRowRange
__global__ void gather_rows_f32_kernel(const float4* __restrict__ x, int64_t n_in, int c4,
                                       const int32_t* __restrict__ rows, int64_t n_out, float4* __restrict__ y,
                                       uint32_t* __restrict__ status) {
    pdl_wait();
    pdl_trigger();
    const int64_t total = n_out * c4;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / c4, q = i - r * c4;
        const int32_t s = __ldg(rows + r);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (s >= 0 && s < n_in)
            v = x[(int64_t)s * c4 + q];
        else if (q == 0)
            atomicOr(status, kErrRowRange);
        y[i] = v;
    }
}
}  // namespace

extern "C" S3DSP_API s3d_status s3dsp_slat_res_block_concat(
    s3dsp_context* ctx, const s3dsp_kmap* kmap, const int32_t* up_rows, uint32_t precision, const float* x_a,
    int64_t cin_a, const float* x_b, int64_t cin_b, int64_t n_in, int64_t cout, const float* norm1_w,
    const float* norm1_b, const void* conv1_w, const float* conv1_b, const float* mod_scale, const float* mod_shift,
    const void* conv2_w, const float* conv2_b, const void* skip_w, const float* skip_b, float* out, char* error,
    uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !kmap || !x_a || !conv1_w || !conv2_w || !out)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    if (x_b ? cin_b <= 0 : cin_b != 0)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "second source and its width disagree");
    const int64_t n = kmap->n_out;
    const int64_t cin = cin_a + cin_b;
    if (cin_a <= 0 || cout <= 0 || n_in <= 0) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "bad shape");
    if (!up_rows && n_in != n) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "n_in != kmap rows");
    if (up_rows && kmap->n_in != n)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "an upsampling block needs the fine rows' own map");
    const bool identity_skip = cin == cout && !x_b && !up_rows;
    if (!identity_skip && !skip_w)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT,
                    "a width change, a concat or an upsample needs the skip Linear (slat_flow_graph.cpp:266-272)");
    if (up_rows && cout % 4)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "upsampled skip rows need cout %% 4 == 0");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    const float eps = 1e-6f;  // gb_layer_norm in res_block (slat_flow_graph.cpp:245-255)
    const bool bf = precision == S3DSP_PREC_BF16;
    const uint32_t hdt = bf ? S3DSP_BF16 : S3DSP_F32;
    const size_t hsz = bf ? 2 : 4;
    Scratch sc(ctx->stream);
    void *h1, *h2;
    float *y1, *skip = nullptr;
    S3DSP_CUDA(sc.get(&h1, hsz * (size_t)(n_in * cin)), "scratch");
    S3DSP_CUDA(sc.get(&h2, hsz * (size_t)(n * cout)), "scratch");
    S3DSP_CUDA(sc.get(&y1, 4 * (size_t)(n * cout)), "scratch");
    // norm1 (affine) -> SiLU over the input rows (coarse rows when upsampling:
    // nearest upsampling repeats rows, so it commutes with the row-wise norm)
    if (x_b)
        S3DSP_TRY(s3dsp_layer_norm_concat(ctx, x_a, cin_a, x_b, cin_b, S3DSP_F32, n_in, eps, norm1_w, norm1_b, nullptr,
                                          nullptr, 1, h1, hdt, error, error_capacity));
    else
        S3DSP_TRY(s3dsp_layer_norm(ctx, x_a, S3DSP_F32, n_in, cin, eps, norm1_w, norm1_b, nullptr, nullptr, 1, h1, hdt,
                                   error, error_capacity));
    // conv1 over the fine map; upsampling reads the coarse rows through the
    // map composed with up_rows (the upsampled tensor is never built)
    s3dsp_kmap* k1 = nullptr;
    if (up_rows) S3DSP_TRY(s3dsp_kmap_compose(ctx, kmap, up_rows, n_in, &k1, error, error_capacity));
    struct KmapGuard {
        s3dsp_context* c;
        s3dsp_kmap* k;
        ~KmapGuard() {
            if (k) s3dsp_kmap_free(c, k);
        }
    } guard{ctx, k1};
    S3DSP_TRY(s3dsp_conv(ctx, k1 ? k1 : kmap, 27, precision, h1, hdt, n_in, cin, 0, conv1_w, conv1_b, nullptr, 0, 0,
                         y1, S3DSP_F32, n, cout, 0, nullptr, nullptr, nullptr, nullptr, 0, error, error_capacity));
    // norm2 (no affine) -> modulate -> SiLU
    S3DSP_TRY(s3dsp_layer_norm(ctx, y1, S3DSP_F32, n, cout, eps, nullptr, nullptr, mod_scale, mod_shift, 1, h2, hdt,
                               error, error_capacity));
    // skip: identity, or the Linear of the (concatenated) input rows, computed
    // on the input rows and then upsampled (the Linear is row-wise too)
    const float* res = x_a;
    if (!identity_skip) {
        const void *sa = x_a, *sb = x_b;
        if (bf) {
            __nv_bfloat16 *xa16, *xb16 = nullptr;
            S3DSP_CUDA(sc.get(&xa16, 2 * (size_t)(n_in * cin_a)), "scratch");
            S3DSP_TRY(s3dsp_convert(ctx, x_a, S3DSP_F32, xa16, S3DSP_BF16, n_in * cin_a, error, error_capacity));
            if (x_b) {
                S3DSP_CUDA(sc.get(&xb16, 2 * (size_t)(n_in * cin_b)), "scratch");
                S3DSP_TRY(s3dsp_convert(ctx, x_b, S3DSP_F32, xb16, S3DSP_BF16, n_in * cin_b, error, error_capacity));
            }
            sa = xa16;
            sb = xb16;
        }
        float* skip_in;
        S3DSP_CUDA(sc.get(&skip_in, 4 * (size_t)(n_in * cout)), "scratch");
        if (x_b)
            S3DSP_TRY(s3dsp_conv_concat(ctx, nullptr, 1, precision, sa, cin_a, sb, cin_b, hdt, n_in, 0, skip_w, skip_b,
                                        nullptr, 0, 0, skip_in, S3DSP_F32, n_in, cout, 0, nullptr, nullptr, nullptr,
                                        nullptr, 0, error, error_capacity));
        else
            S3DSP_TRY(s3dsp_conv(ctx, nullptr, 1, precision, sa, hdt, n_in, cin, 0, skip_w, skip_b, nullptr, 0, 0,
                                 skip_in, S3DSP_F32, n_in, cout, 0, nullptr, nullptr, nullptr, nullptr, 0, error,
                                 error_capacity));
        skip = skip_in;
        if (up_rows) {
            S3DSP_CUDA(sc.get(&skip, 4 * (size_t)(n * cout)), "scratch");
            const int c4 = (int)(cout / 4);
            int64_t g = (n * c4 + 255) / 256;
            if (g > (int64_t)ctx->sm_count * 16) g = (int64_t)ctx->sm_count * 16;
            S3DSP_CUDA(launch_pdl(gather_rows_f32_kernel, dim3((unsigned)(g < 1 ? 1 : g)), dim3(256), 0, ctx->stream,
                                  reinterpret_cast<const float4*>(skip_in), n_in, c4, up_rows, n,
                                  reinterpret_cast<float4*>(skip), ctx->d_status),
                       "gather_rows_f32_kernel");
        }
        res = skip;
    }
    return s3dsp_conv(ctx, kmap, 27, precision, h2, hdt, n, cout, 0, conv2_w, conv2_b, res, S3DSP_F32, 0, out,
                      S3DSP_F32, n, cout, 0, nullptr, nullptr, nullptr, nullptr, 0, error, error_capacity);
}

// ---------------------------------------------------------------------------
// Host-buffer entry points: what the reference's per-level code does with its
// Backend (upload coords + features, run, read back: session.cpp:927-962), as
// one call. Weights stay device-resident (packed once at model load).
// ---------------------------------------------------------------------------
namespace {
// host coords + features in, the block, host output out, on the context's
// stream; `wait` = synchronise and report device-detected errors before
// returning (the synchronous entry point), else return once queued
// The host-buffer block on a context with S3DSP_CONTEXT_COPY_STREAMS: staging
// slot j % 3 for call j; copies in on the copy-in stream, the tables and the
// block on the context's stream, the copy out on the copy-out stream, so that
// call j + 1's upload and call j - 1's download run beside call j's kernels.
// Returns with the work queued.
s3d_status res_block_gn_host_piped(s3dsp_context* ctx, uint32_t precision, const int32_t* h_coords, int64_t n,
                                   const float* h_x, int64_t c, const void* w1, const float* b1, const float* gamma,
                                   const float* beta, const void* w2, const float* b2, int32_t groups, float eps,
                                   float* h_out, char* error, uint64_t error_capacity) {
    s3dsp_host_pipe* p = ctx->pipe;
    s3dsp_host_pipe::Slot& s = p->slots[p->calls % s3dsp_host_pipe::kSlots];
    const size_t cb = 16 * (size_t)n, xb = 4 * (size_t)(n * c), ob = 4 * (size_t)(n * c);
    // the slot's previous call must have consumed its inputs before they are overwritten
    if (s.used) S3DSP_CUDA(cudaStreamWaitEvent(p->copy_in, s.comp_done, 0), "cudaStreamWaitEvent");
    if (s.coords_bytes < cb || s.x_bytes < xb || s.out_bytes < ob) {
        // larger buffers: the old ones go once the slot's previous output is copied out
        if (s.used) S3DSP_CUDA(cudaStreamWaitEvent(p->copy_in, s.out_done, 0), "cudaStreamWaitEvent");
        void** bufs[3] = {&s.d_coords, &s.d_x, &s.d_out};
        size_t* have[3] = {&s.coords_bytes, &s.x_bytes, &s.out_bytes};
        const size_t want[3] = {cb, xb, ob};
        for (int i = 0; i < 3; ++i) {
            if (*have[i] >= want[i]) continue;
            if (*bufs[i]) S3DSP_CUDA(cudaFreeAsync(*bufs[i], p->copy_in), "cudaFreeAsync");
            *bufs[i] = nullptr;
            *have[i] = 0;
            S3DSP_CUDA(s3dsp::malloc_async(bufs[i], want[i], p->copy_in), "staging allocation");
            *have[i] = want[i];
        }
    }
    S3DSP_CUDA(cudaMemcpyAsync(s.d_coords, h_coords, cb, cudaMemcpyHostToDevice, p->copy_in), "H2D coords");
    S3DSP_CUDA(cudaMemcpyAsync(s.d_x, h_x, xb, cudaMemcpyHostToDevice, p->copy_in), "H2D features");
    S3DSP_CUDA(cudaEventRecord(s.in_done, p->copy_in), "cudaEventRecord");
    S3DSP_CUDA(cudaStreamWaitEvent(ctx->stream, s.in_done, 0), "cudaStreamWaitEvent");
    // d_out is rewritten only after the slot's previous output has been copied out
    if (s.used) S3DSP_CUDA(cudaStreamWaitEvent(ctx->stream, s.out_done, 0), "cudaStreamWaitEvent");
    s3dsp_hash* h = nullptr;
    s3dsp_kmap* k = nullptr;
    s3d_status st = s3dsp_hash_build(ctx, static_cast<const int32_t*>(s.d_coords), n, 0, &h, error, error_capacity);
    if (st == S3D_OK) st = s3dsp_kmap_build_subm3(ctx, h, &k, error, error_capacity);
    if (st == S3D_OK)
        st = s3dsp_res_block_gn(ctx, k, precision, static_cast<const float*>(s.d_x), n, c, w1, b1, gamma, beta, w2,
                                b2, groups, eps, static_cast<float*>(s.d_out), error, error_capacity);
    s3dsp_kmap_free(ctx, k);
    s3dsp_hash_free(ctx, h);
    // the slot's events are recorded whatever happened, so later calls order correctly
    cudaError_t e = cudaEventRecord(s.comp_done, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(p->copy_out, s.comp_done, 0);
    if (e == cudaSuccess && st == S3D_OK) {
        e = cudaMemcpyAsync(h_out, s.d_out, ob, cudaMemcpyDeviceToHost, p->copy_out);
        if (e != cudaSuccess) st = cuda_fail(error, error_capacity, e, "D2H output");
    }
    const cudaError_t e2 = cudaEventRecord(s.out_done, p->copy_out);
    if (e == cudaSuccess) e = e2;
    s.used = true;
    ++p->calls;
    if (st == S3D_OK && e != cudaSuccess) st = cuda_fail(error, error_capacity, e, "copy-stream ordering");
    return st;
}

s3d_status res_block_gn_host_impl(s3dsp_context* ctx, uint32_t precision, const int32_t* h_coords, int64_t n,
                                  const float* h_x, int64_t c, const void* w1, const float* b1, const float* gamma,
                                  const float* beta, const void* w2, const float* b2, int32_t groups, float eps,
                                  float* h_out, bool wait, char* error, uint64_t error_capacity) {
    if (!ctx || !h_coords || !h_x || !h_out || n <= 0 || c <= 0)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "bad argument");
    if (!wait && !(ctx->flags & S3DSP_CONTEXT_DEFERRED_CHECKS))
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT,
                    "the queued form needs a context with S3DSP_CONTEXT_DEFERRED_CHECKS");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    if (ctx->pipe) {
        s3d_status s = res_block_gn_host_piped(ctx, precision, h_coords, n, h_x, c, w1, b1, gamma, beta, w2, b2,
                                               groups, eps, h_out, error, error_capacity);
        if (s == S3D_OK && wait) {
            cudaError_t e = pipe_join(ctx);
            if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
            if (e != cudaSuccess) s = cuda_fail(error, error_capacity, e, "cudaStreamSynchronize");
            if (s == S3D_OK && (ctx->flags & S3DSP_CONTEXT_DEFERRED_CHECKS)) s = check_status(ctx, error, error_capacity);
        }
        return s;
    }
    Scratch sc(ctx->stream);
    int32_t* d_coords;
    float *d_x, *d_out;
    S3DSP_CUDA(sc.get(&d_coords, 16 * (size_t)n), "scratch");
    S3DSP_CUDA(sc.get(&d_x, 4 * (size_t)(n * c)), "scratch");
    S3DSP_CUDA(sc.get(&d_out, 4 * (size_t)(n * c)), "scratch");
    S3DSP_CUDA(cudaMemcpyAsync(d_coords, h_coords, 16 * (size_t)n, cudaMemcpyHostToDevice, ctx->stream), "H2D coords");
    S3DSP_CUDA(cudaMemcpyAsync(d_x, h_x, 4 * (size_t)(n * c), cudaMemcpyHostToDevice, ctx->stream), "H2D features");
    s3dsp_hash* h = nullptr;
    S3DSP_TRY(s3dsp_hash_build(ctx, d_coords, n, 0, &h, error, error_capacity));
    s3dsp_kmap* k = nullptr;
    s3d_status s = s3dsp_kmap_build_subm3(ctx, h, &k, error, error_capacity);
    if (s == S3D_OK)
        s = s3dsp_res_block_gn(ctx, k, precision, d_x, n, c, w1, b1, gamma, beta, w2, b2, groups, eps, d_out, error,
                               error_capacity);
    if (s == S3D_OK) {
        const cudaError_t e = cudaMemcpyAsync(h_out, d_out, 4 * (size_t)(n * c), cudaMemcpyDeviceToHost, ctx->stream);
        if (e != cudaSuccess) s = cuda_fail(error, error_capacity, e, "D2H output");
    }
    s3dsp_kmap_free(ctx, k);
    s3dsp_hash_free(ctx, h);
    if (s == S3D_OK && wait) {
        const cudaError_t e = cudaStreamSynchronize(ctx->stream);
        if (e != cudaSuccess) s = cuda_fail(error, error_capacity, e, "cudaStreamSynchronize");
        if (s == S3D_OK && (ctx->flags & S3DSP_CONTEXT_DEFERRED_CHECKS)) s = check_status(ctx, error, error_capacity);
    }
    return s;
}
}  // namespace

extern "C" S3DSP_API s3d_status s3dsp_res_block_gn_host(s3dsp_context* ctx, uint32_t precision,
                                                        const int32_t* h_coords, int64_t n, const float* h_x, int64_t c,
                                                        const void* w1, const float* b1, const float* gamma,
                                                        const float* beta, const void* w2, const float* b2,
                                                        int32_t groups, float eps, float* h_out, char* error,
                                                        uint64_t error_capacity) {
    clear_error(error, error_capacity);
    return res_block_gn_host_impl(ctx, precision, h_coords, n, h_x, c, w1, b1, gamma, beta, w2, b2, groups, eps, h_out,
                                  true, error, error_capacity);
}

extern "C" S3DSP_API s3d_status s3dsp_res_block_gn_host_queued(s3dsp_context* ctx, uint32_t precision,
                                                               const int32_t* h_coords, int64_t n, const float* h_x,
                                                               int64_t c, const void* w1, const float* b1,
                                                               const float* gamma, const float* beta, const void* w2,
                                                               const float* b2, int32_t groups, float eps,
                                                               float* h_out, char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    return res_block_gn_host_impl(ctx, precision, h_coords, n, h_x, c, w1, b1, gamma, beta, w2, b2, groups, eps, h_out,
                                  false, error, error_capacity);
}

extern "C" S3DSP_API s3d_status s3dsp_mesh_upsample_level_host(
    s3dsp_context* ctx, uint32_t precision, const int32_t* h_parent_coords, int64_t np, const float* h_x, int64_t cin,
    int64_t cout, const float* gn1_w, const float* gn1_b, const void* conv1_w, const float* conv1_b,
    const float* gn2_w, const float* gn2_b, const void* conv2_w, const float* conv2_b, const void* skip_w,
    const float* skip_b, int32_t* h_child_coords, float* h_out, char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !h_parent_coords || !h_x || !h_child_coords || !h_out || np <= 0)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "bad argument");
    if (np > INT32_MAX / 8) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "parent count exceeds INT32_MAX/8");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    const int64_t nc = 8 * np;
    Scratch sc(ctx->stream);
    int32_t *d_pc, *d_cc;
    float *d_x, *d_out;
    S3DSP_CUDA(sc.get(&d_pc, 16 * (size_t)np), "scratch");
    S3DSP_CUDA(sc.get(&d_cc, 16 * (size_t)nc), "scratch");
    S3DSP_CUDA(sc.get(&d_x, 4 * (size_t)(np * cin)), "scratch");
    S3DSP_CUDA(sc.get(&d_out, 4 * (size_t)(nc * cout)), "scratch");
    S3DSP_CUDA(cudaMemcpyAsync(d_pc, h_parent_coords, 16 * (size_t)np, cudaMemcpyHostToDevice, ctx->stream), "H2D coords");
    S3DSP_CUDA(cudaMemcpyAsync(d_x, h_x, 4 * (size_t)(np * cin), cudaMemcpyHostToDevice, ctx->stream), "H2D features");
    s3dsp_hash* h = nullptr;
    S3DSP_TRY(s3dsp_hash_build(ctx, d_pc, np, 1, &h, error, error_capacity));
    s3d_status s = s3dsp_mesh_upsample_level(ctx, h, precision, d_x, cin, cout, gn1_w, gn1_b, conv1_w, conv1_b, gn2_w,
                                             gn2_b, conv2_w, conv2_b, skip_w, skip_b, d_cc, d_out, error,
                                             error_capacity);
    if (s == S3D_OK) {
        cudaError_t e = cudaMemcpyAsync(h_child_coords, d_cc, 16 * (size_t)nc, cudaMemcpyDeviceToHost, ctx->stream);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(h_out, d_out, 4 * (size_t)(nc * cout), cudaMemcpyDeviceToHost, ctx->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
        if (e != cudaSuccess) s = cuda_fail(error, error_capacity, e, "readback");
    }
    s3dsp_hash_free(ctx, h);
    if (s == S3D_OK && (ctx->flags & S3DSP_CONTEXT_DEFERRED_CHECKS)) s = check_status(ctx, error, error_capacity);
    return s;
}
