// s3dsp_conv: argument validation and dispatch to the F32-strict (FP32 FMA)
// or BF16 (tcgen05) implicit-gather kernels.
#include "s3dsp_internal.h"

using namespace s3dsp;

namespace {

// BF16 kernel choice by estimated time, in units of one wave of 128-row
// tiles (every SM running one full tile; column blocks of 256 count as
// tiles). 128-row tiles: ceil(tiles / SMs) waves. Stream-K (256-row tiles
// split evenly over the SMs): a fixed ~0.55 wave for the split-tile fix-up
// and pipeline refills, plus 1.525 / kvol of a wave per (256-row tile,
// offset) unit and SM. Split-K pairs (one cluster of two CTAs per 256-row
// tile, half the offsets each): 0.95 of a wave per wave of pairs. Fitted to
// B200 sweeps of 32^3..256^3 shells at C = 64..1024 (2k-242k rows): pairs
// win while the pairs fill one or two waves (config 2, 15k rows: 84 vs 88 us
// for 128-row tiles), stream-K for wide layers and for a thin last wave
// (155 tiles: 2 waves vs ~1.35). Maps with few offsets (linear layers)
// always use 128-row tiles.
enum class Bf16Kernel { kTile128, kStreamK128, kStreamK256, kSplit256, kHalo };

// halo: the one-source layers the per-tile halo kernel takes (cin <= 256,
// cout <= 128 in one column tile, kvol <= 27)
Bf16Kernel pick_bf16_kernel(const s3dsp_context* ctx, int64_t n_out, int32_t kvol, int64_t cin, int64_t cout,
                            int in_shift, bool two_sources, uint32_t flags) {
    int hs = 0, hc = 0, hp = 0;
    const bool halo_ok = !two_sources && kvol > 1 && cin <= 256 && cout <= 128 &&
                         conv_halo_plan((int)cin, (int)cout, kvol, in_shift, &hs, &hc, &hp);
    if ((flags & S3DSP_CONV_HALO) && halo_ok) return Bf16Kernel::kHalo;
    if (flags & (S3DSP_CONV_TILE128 | S3DSP_CONV_CTA_PAIR)) return Bf16Kernel::kTile128;
    if (flags & S3DSP_CONV_STREAM_K128) return Bf16Kernel::kStreamK128;
    if (flags & S3DSP_CONV_STREAM_K) return Bf16Kernel::kStreamK256;
    if (flags & S3DSP_CONV_SPLIT_PAIRS) return Bf16Kernel::kSplit256;
    if (kvol < 8) return Bf16Kernel::kTile128;
    const int64_t sm = ctx->sm_count;
    // layers of at most 64 output channels whose halo fits two CTAs per SM, at
    // least one wave of 128-row tiles: the halo kernel (B200, twice-subdivided
    // 64^3 shell: C = 64 at 970k rows 852 vs 1,150 us for stream-K, the
    // 128 -> 64 subdivide conv 1,287 vs 1,572 us; 121k rows 125 vs 151 us)
    if (halo_ok && hp == 2 && cout <= 64 && (n_out + 127) / 128 >= sm) return Bf16Kernel::kHalo;
    const int64_t nnb = ((cout + 15) / 16 * 16) / tc_pick_bn((int)cout);  // column blocks
    const int64_t tiles = (n_out + 127) / 128 * nnb;
    const int64_t work = (n_out + 255) / 256 * nnb;  // 256-row work tiles
    const double waves128 = (double)((tiles + sm - 1) / sm);
    const double est_sk = 0.55 + ((double)(work * kvol) / (double)sm) * 1.525 / kvol;
    const double est_pairs = 0.95 * (double)((2 * work + sm - 1) / sm);
    if (est_pairs <= est_sk && est_pairs < waves128) return Bf16Kernel::kSplit256;
    return est_sk < 0.95 * waves128 ? Bf16Kernel::kStreamK256 : Bf16Kernel::kTile128;
}

const char* bf16_kernel_name(Bf16Kernel k) {
    return k == Bf16Kernel::kTile128      ? "conv_tc_kernel"
           : k == Bf16Kernel::kStreamK128 ? "conv_sk_kernel<128>"
           : k == Bf16Kernel::kSplit256   ? "conv_sk_kernel<256>:pairs"
           : k == Bf16Kernel::kHalo       ? "conv_halo_kernel"
                                          : "conv_sk_kernel<256>";
}

}  // namespace

extern "C" S3DSP_API const char* s3dsp_conv_kernel_shift(const s3dsp_context* ctx, int64_t n_out, int32_t kvol,
                                                         int64_t cin, int64_t cout, int32_t in_shift,
                                                         uint32_t precision, uint32_t flags) {
    if (!ctx || in_shift < 0 || in_shift > 8) return nullptr;
    if (precision == S3DSP_PREC_F32_STRICT) return "conv_f32_kernel";
    if (precision == S3DSP_PREC_F32_3XTF32) return "conv_tc_kernel<tf32x3>";
    if (precision != S3DSP_PREC_BF16) return nullptr;
    if (cout <= 0) return nullptr;
    return bf16_kernel_name(pick_bf16_kernel(ctx, n_out, kvol, cin, cout, in_shift, false, flags));
}

extern "C" S3DSP_API const char* s3dsp_conv_kernel(const s3dsp_context* ctx, int64_t n_out, int32_t kvol, int64_t cin,
                                                   int64_t cout, uint32_t precision, uint32_t flags) {
    return s3dsp_conv_kernel_shift(ctx, n_out, kvol, cin, cout, 0, precision, flags);
}

namespace {

// s3dsp_conv and s3dsp_conv_concat: in_b == nullptr is one source (cin_a == cin)
s3d_status conv_impl(s3dsp_context* ctx, const s3dsp_kmap* kmap, int32_t kvol, uint32_t precision, const void* in,
                     const void* in_b, int64_t cin_a, uint32_t in_dtype, int64_t n_in, int64_t cin, int32_t in_shift,
                     const void* weight, const float* bias, const void* residual, uint32_t res_dtype,
                     int32_t res_shift, void* out, uint32_t out_dtype, int64_t n_out, int64_t cout, uint32_t flags,
                     const float* pro_sub, const float* pro_mul, const float* pro_add, double* gn_partials,
                     int32_t gn_groups, char* error, uint64_t error_capacity) {
    if (!ctx || !in || !weight || !out) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    if (kmap) {
        if (kvol != kmap->kvol)
            return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "kvol %d != kmap kvol %d", kvol, kmap->kvol);
        if (n_out != kmap->n_out)
            return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "n_out %lld != kmap rows %lld", (long long)n_out,
                        (long long)kmap->n_out);
    } else if (kvol != 1) {
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "identity conv (kmap NULL) needs kvol 1");
    }
    if (n_out < 0 || n_in < 0 || cin <= 0 || cout <= 0 || cin > 65536 || cout > 65536)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "bad shape");
    if (in_b && (cin_a <= 0 || cin_a >= cin))
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "concat split %lld outside (0, %lld)",
                    (long long)cin_a, (long long)cin);
    if (n_out == 0) return S3D_OK;
    if (n_out > (1ll << 31) - 128) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "n_out too large");
    if (in_shift < 0 || in_shift > 8 || res_shift < 0 || res_shift > 8)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "shift out of range");
    if (!kmap && ((n_out - 1) >> in_shift) >= n_in)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "identity conv reads past n_in");
    // every gathered row index is < kmap->n_in, read as (index >> in_shift)
    if (kmap && kmap->n_in > 0 && ((kmap->n_in - 1) >> in_shift) >= n_in)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT,
                    "kmap gathers rows up to %lld (>> %d) but the input has %lld rows",
                    (long long)kmap->n_in - 1, in_shift, (long long)n_in);
    if (!dtype_ok(out_dtype) || (residual && !dtype_ok(res_dtype)))
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "bad dtype");
    if (gn_partials && (gn_groups <= 0 || gn_groups > 64 || cout % gn_groups))
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "GroupNorm groups %d must divide cout %lld (<= 64)",
                    gn_groups, (long long)cout);
    if ((flags & S3DSP_EPI_SILU) && (flags & S3DSP_EPI_GELU))
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "SiLU and GELU epilogues are exclusive");
    if ((flags & S3DSP_PRO_AFFINE_SILU) && (!pro_sub || !pro_mul || !pro_add))
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "prologue arrays missing");
    const int ca = (int)(in_b ? cin_a : cin);
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");

    cudaError_t e;
    if (precision == S3DSP_PREC_F32_STRICT) {
        if (in_dtype != S3DSP_F32)
            return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "F32_STRICT needs f32 input");
        if (cin % 4 || ca % 4 || ((uintptr_t)in & 15) || ((uintptr_t)in_b & 15))
            return fail(error, error_capacity, S3D_INVALID_ARGUMENT,
                        "F32_STRICT needs cin %% 4 == 0 (each source) and 16-byte rows");
        e = launch_conv_f32(ctx, kmap, kvol, (const float*)in, (const float*)in_b, ca, n_in, (int)cin, in_shift,
                            (const float*)weight, bias, residual, res_dtype, res_shift, out, out_dtype, n_out,
                            (int)cout, flags, pro_sub, pro_mul, pro_add, gn_partials, gn_groups);
        if (e != cudaSuccess) return cuda_fail(error, error_capacity, e, "conv_f32_kernel");
        return S3D_OK;
    }
    if (precision == S3DSP_PREC_BF16) {
        if (in_dtype != S3DSP_BF16)
            return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "BF16 precision needs bf16 input");
        if (flags & S3DSP_PRO_AFFINE_SILU)
            return fail(error, error_capacity, S3D_INVALID_ARGUMENT,
                        "BF16 conv takes pre-normalised input (use s3dsp_channel_affine)");
        if (cin % 8 || ca % 8 || ((uintptr_t)in & 15) || ((uintptr_t)in_b & 15) || ((uintptr_t)weight & 15) ||
            ((uintptr_t)out & 15) || ((uintptr_t)residual & 15))
            return fail(error, error_capacity, S3D_INVALID_ARGUMENT,
                        "BF16 needs cin %% 8 == 0 (each source) and 16-byte aligned in/weight/out/residual");
        s3d_status st = S3D_OK;
        const Bf16Kernel kern = pick_bf16_kernel(ctx, n_out, kvol, cin, cout, in_shift, in_b != nullptr, flags);
        if (kern == Bf16Kernel::kHalo)
            e = launch_conv_halo(ctx, kmap, kvol, (const __nv_bfloat16*)in, (int)cin, in_shift,
                                 (const __nv_bfloat16*)weight, bias, residual, res_dtype, res_shift, out, out_dtype,
                                 n_out, (int)cout, flags, gn_partials, gn_groups, error, error_capacity, &st);
        else if (kern == Bf16Kernel::kTile128)
            e = launch_conv_tc(ctx, kmap, kvol, (const __nv_bfloat16*)in, (const __nv_bfloat16*)in_b, ca, n_in,
                               (int)cin, in_shift, (const __nv_bfloat16*)weight, bias, residual, res_dtype, res_shift,
                               out, out_dtype, n_out, (int)cout, flags, gn_partials, gn_groups, error,
                               error_capacity, &st);
        else
            e = launch_conv_sk(ctx, kmap, kvol, (const __nv_bfloat16*)in, (const __nv_bfloat16*)in_b, ca, n_in,
                               (int)cin, in_shift, (const __nv_bfloat16*)weight, bias, residual, res_dtype, res_shift,
                               out, out_dtype, n_out, (int)cout, flags, gn_partials, gn_groups,
                               kern == Bf16Kernel::kStreamK128 ? 128 : 256, kern == Bf16Kernel::kSplit256 ? 2 : 1,
                               error, error_capacity, &st);
        if (st != S3D_OK) return st;
        if (e != cudaSuccess) return cuda_fail(error, error_capacity, e, bf16_kernel_name(kern));
        return S3D_OK;
    }
    if (precision == S3DSP_PREC_F32_3XTF32) {
        if (in_dtype != S3DSP_F32)
            return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "3XTF32 precision needs f32 input");
        if (flags & (S3DSP_PRO_AFFINE_SILU | S3DSP_CONV_CTA_PAIR))
            return fail(error, error_capacity, S3D_INVALID_ARGUMENT,
                        "3XTF32 conv takes pre-normalised input and runs without CTA pairs");
        if (cin % 4 || ca % 4 || ((uintptr_t)in & 15) || ((uintptr_t)in_b & 15) || ((uintptr_t)weight & 15) ||
            ((uintptr_t)out & 15) || ((uintptr_t)residual & 15))
            return fail(error, error_capacity, S3D_INVALID_ARGUMENT,
                        "3XTF32 needs cin %% 4 == 0 (each source) and 16-byte aligned in/weight/out/residual");
        // each source split once into TF32 high parts and remainders (stream-ordered scratch)
        const size_t nel_a = (size_t)n_in * (size_t)ca;
        const size_t nel_b = in_b ? (size_t)n_in * (size_t)(cin - ca) : 0;
        const size_t nel = nel_a + nel_b;
        float* split = nullptr;
        S3DSP_CUDA(s3dsp::malloc_async(&split, 8 * (nel > 0 ? nel : 1), ctx->stream), "3xTF32 split buffer");
        float* hi_a = split;
        float* lo_a = split + nel_a;
        float* hi_b = split + 2 * nel_a;
        float* lo_b = hi_b + nel_b;
        e = split_tf32(ctx, (const float*)in, (int64_t)nel_a, hi_a, lo_a);
        if (e == cudaSuccess && in_b) e = split_tf32(ctx, (const float*)in_b, (int64_t)nel_b, hi_b, lo_b);
        s3d_status st = S3D_OK;
        if (e == cudaSuccess)
            e = launch_conv_tf32x3(ctx, kmap, kvol, hi_a, lo_a, in_b ? hi_b : nullptr, in_b ? lo_b : nullptr, ca,
                                   (int)cin, in_shift, (const float*)weight, bias, residual, res_dtype, res_shift, out,
                                   out_dtype, n_out, (int)cout, flags, gn_partials, gn_groups, error, error_capacity,
                                   &st);
        cudaFreeAsync(split, ctx->stream);
        if (st != S3D_OK) return st;
        if (e != cudaSuccess) return cuda_fail(error, error_capacity, e, "conv_tc_kernel<tf32x3>");
        return S3D_OK;
    }
    return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "unknown precision %u", precision);
}

}  // namespace

extern "C" S3DSP_API s3d_status s3dsp_conv(s3dsp_context* ctx, const s3dsp_kmap* kmap, int32_t kvol,
                                           uint32_t precision, const void* in, uint32_t in_dtype, int64_t n_in,
                                           int64_t cin, int32_t in_shift, const void* weight, const float* bias,
                                           const void* residual, uint32_t res_dtype, int32_t res_shift, void* out,
                                           uint32_t out_dtype, int64_t n_out, int64_t cout, uint32_t flags,
                                           const float* pro_sub, const float* pro_mul, const float* pro_add,
                                           double* gn_partials, int32_t gn_groups, char* error,
                                           uint64_t error_capacity) {
    clear_error(error, error_capacity);
    return conv_impl(ctx, kmap, kvol, precision, in, nullptr, cin, in_dtype, n_in, cin, in_shift, weight, bias,
                     residual, res_dtype, res_shift, out, out_dtype, n_out, cout, flags, pro_sub, pro_mul, pro_add,
                     gn_partials, gn_groups, error, error_capacity);
}

extern "C" S3DSP_API s3d_status s3dsp_conv_concat(s3dsp_context* ctx, const s3dsp_kmap* kmap, int32_t kvol,
                                                  uint32_t precision, const void* in_a, int64_t cin_a,
                                                  const void* in_b, int64_t cin_b, uint32_t in_dtype, int64_t n_in,
                                                  int32_t in_shift, const void* weight, const float* bias,
                                                  const void* residual, uint32_t res_dtype, int32_t res_shift,
                                                  void* out, uint32_t out_dtype, int64_t n_out, int64_t cout,
                                                  uint32_t flags, const float* pro_sub, const float* pro_mul,
                                                  const float* pro_add, double* gn_partials, int32_t gn_groups,
                                                  char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!in_b || cin_b <= 0) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "second source missing");
    return conv_impl(ctx, kmap, kvol, precision, in_a, in_b, cin_a, in_dtype, n_in, cin_a + cin_b, in_shift, weight,
                     bias, residual, res_dtype, res_shift, out, out_dtype, n_out, cout, flags, pro_sub, pro_mul,
                     pro_add, gn_partials, gn_groups, error, error_capacity);
}
