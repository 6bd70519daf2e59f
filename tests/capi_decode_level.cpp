// A C++ host of the s3dsp C ABI that includes only include/s3dsp.h: the shape
// of the code sam3d.cpp's decode_object_mesh would run per level
// (src/objects_runtime/session.cpp:895-996: upload the level's inputs, run the
// graph, read the result back, :927-962), calling the library step by step
// the way INTEGRATION.md sketches it instead of building GGML graphs.
//
//   capi_decode_level <dir>
//
// Inputs, SAMT files in <dir> (written by tests/test_capi_cpp_gpu.py):
//   level_parents.samt [np, 4] i32, level_x.samt [np, cin] f32, and the
//   level's gn1_w gn1_b conv1_w (27, cout*cin) conv1_b gn2_w gn2_b conv2_w
//   (27, cout*cout) conv2_b skip_w (cout, cin) skip_b as level_<name>.samt;
//   block_coords.samt [n, 4] i32, block_x.samt [n, c] f32, and block_w1
//   (c, 27*c) block_b1 block_gamma block_beta block_w2 block_b2.
// Outputs, SAMT files in <dir>:
//   out_level_child_coords.samt [8np, 4] i32, out_level.samt [8np, cout] f32
//   (one MeshUpsampleGraph level, mesh_decoder_graph.cpp:42-132, BF16);
//   out_block.samt [n, c] f32 (the config-2 residual block, BF16).
// Exit status 0 on success; otherwise the failing call and its message.
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

#include "s3dsp.h"

namespace {

char g_err[512];
const char* g_what = "";

bool ok(s3d_status st, const char* what) {
    if (st == S3D_OK) return true;
    g_what = what;
    std::fprintf(stderr, "%s failed (status %u): %s\n", what, st, g_err);
    return false;
}
#define CALL(expr) \
    do {                                   \
        if (!ok((expr), #expr)) return 1;  \
    } while (0)

// A host tensor read from a SAMT file (the reference's raw tensor format,
// common.cpp:59-119): shape in numpy order, bytes.
struct HostTensor {
    std::vector<int64_t> shape;
    std::vector<unsigned char> bytes;
    int64_t dim(int i) const { return shape[(size_t)i]; }
    const void* data() const { return bytes.data(); }
};

bool read_samt(const std::string& path, HostTensor* t) {
    int32_t nd = 0, type = 0;
    int64_t ne[8] = {};
    uint64_t nbytes = 0;
    if (!ok(s3dsp_samt_info(path.c_str(), &nd, ne, &type, &nbytes, g_err, sizeof g_err), path.c_str())) return false;
    t->shape.assign((size_t)nd, 0);
    for (int i = 0; i < nd; ++i) t->shape[(size_t)i] = ne[nd - 1 - i];
    t->bytes.resize(nbytes);
    return ok(s3dsp_samt_read(path.c_str(), t->bytes.data(), nbytes, g_err, sizeof g_err), path.c_str());
}

bool write_samt(const std::string& path, const std::vector<int64_t>& shape, int32_t ggml_type, const void* data,
                uint64_t nbytes) {
    std::vector<int64_t> ne(shape.rbegin(), shape.rend());
    return ok(s3dsp_samt_write(path.c_str(), (int32_t)ne.size(), ne.data(), ggml_type, data, nbytes, g_err,
                               sizeof g_err),
              path.c_str());
}

constexpr int32_t kGgmlF32 = 0, kGgmlI32 = 26;

// device buffers owned by this host (Backend::alloc's counterpart), freed at exit
struct Buffers {
    s3dsp_context* ctx = nullptr;
    std::vector<void*> ptrs;
    ~Buffers() {
        for (void* p : ptrs) s3dsp_device_free(ctx, p);
    }
    void* get(uint64_t bytes) {
        void* p = nullptr;
        if (!ok(s3dsp_device_alloc(ctx, bytes, &p, g_err, sizeof g_err), "s3dsp_device_alloc")) return nullptr;
        ptrs.push_back(p);
        return p;
    }
    void* upload(const HostTensor& t) {
        void* p = get(t.bytes.size());
        if (p && !ok(s3dsp_copy_to_device(ctx, p, t.data(), t.bytes.size(), g_err, sizeof g_err),
                     "s3dsp_copy_to_device"))
            return nullptr;
        return p;
    }
    // a weight packed for `precision` from its GGUF-layout host tensor
    void* pack(const HostTensor& w, uint32_t layout, int32_t kvol, int64_t cin, int64_t cout, uint32_t precision) {
        void* p = get((uint64_t)s3dsp_weights_packed_bytes(precision, kvol, cin, cout));
        if (p && !ok(s3dsp_weights_pack(ctx, w.data(), S3DSP_F32, 1, layout, kvol, cin, cout, precision, p, g_err,
                                        sizeof g_err),
                     "s3dsp_weights_pack"))
            return nullptr;
        return p;
    }
};

#define NEED(p)                                                   \
    do {                                                          \
        if (!(p)) return 1;                                       \
    } while (0)

// One mesh upsample level, BF16: GN1 + SiLU on the parents, conv1 over the
// 8 children gathering parent rows (in_shift 3: repeat_children without the
// copy) with GN2 partial sums from its epilogue, GN2 + SiLU, conv2, + the 1x1
// skip of the parents broadcast to their children (res_shift 3).
int run_level(s3dsp_context* ctx, Buffers& buf, const std::string& dir) {
    const uint32_t P = S3DSP_PREC_BF16;
    HostTensor parents, x, gn1_w, gn1_b, conv1_w, conv1_b, gn2_w, gn2_b, conv2_w, conv2_b, skip_w, skip_b;
    const std::pair<const char*, HostTensor*> files[] = {
        {"level_parents", &parents}, {"level_x", &x},           {"level_gn1_w", &gn1_w},     {"level_gn1_b", &gn1_b},
        {"level_conv1_w", &conv1_w}, {"level_conv1_b", &conv1_b}, {"level_gn2_w", &gn2_w},   {"level_gn2_b", &gn2_b},
        {"level_conv2_w", &conv2_w}, {"level_conv2_b", &conv2_b}, {"level_skip_w", &skip_w}, {"level_skip_b", &skip_b}};
    for (const auto& f : files)
        if (!read_samt(dir + "/" + f.first + ".samt", f.second)) return 1;
    const int64_t np = parents.dim(0), cin = x.dim(1), cout = conv1_b.dim(0), nc = 8 * np;
    const int32_t groups = 32;
    const float eps = 1e-5f;
    // upload the level's inputs (set_input_i32 / set_input_f32) and pack the weights once
    void* d_parents = buf.upload(parents);
    void* d_x = buf.upload(x);
    NEED(d_parents && d_x);
    void* d_gn1_w = buf.upload(gn1_w);
    void* d_gn1_b = buf.upload(gn1_b);
    void* d_gn2_w = buf.upload(gn2_w);
    void* d_gn2_b = buf.upload(gn2_b);
    void* d_conv1_b = buf.upload(conv1_b);
    void* d_conv2_b = buf.upload(conv2_b);
    void* d_skip_b = buf.upload(skip_b);
    NEED(d_gn1_w && d_gn1_b && d_gn2_w && d_gn2_b && d_conv1_b && d_conv2_b && d_skip_b);
    void* d_w1 = buf.pack(conv1_w, S3DSP_LAYOUT_MESH_PACKED, 27, cin, cout, P);
    void* d_w2 = buf.pack(conv2_w, S3DSP_LAYOUT_MESH_PACKED, 27, cout, cout, P);
    void* d_ws = buf.pack(skip_w, S3DSP_LAYOUT_LINEAR, 1, cin, cout, P);
    NEED(d_w1 && d_w2 && d_ws);
    // scratch
    const int64_t gmax = nc > np ? nc : np;
    auto* d_part = static_cast<double*>(buf.get(8 * (uint64_t)s3dsp_gn_partials_count(gmax, 1, groups)));
    auto* d_aff = static_cast<float*>(buf.get(4 * 3 * (uint64_t)(cin > cout ? cin : cout)));
    void* d_xb = buf.get(2 * (uint64_t)(np * cin));
    void* d_h1 = buf.get(2 * (uint64_t)(np * cin));
    void* d_y1 = buf.get(2 * (uint64_t)(nc * cout));
    void* d_h2 = buf.get(2 * (uint64_t)(nc * cout));
    auto* d_skip = static_cast<float*>(buf.get(4 * (uint64_t)(np * cout)));
    auto* d_out = static_cast<float*>(buf.get(4 * (uint64_t)(nc * cout)));
    auto* d_child = static_cast<int32_t*>(buf.get(16 * (uint64_t)nc));
    NEED(d_part && d_aff && d_xb && d_h1 && d_y1 && d_h2 && d_skip && d_out && d_child);
    const int64_t cm = cin > cout ? cin : cout;
    float *sub = d_aff, *mul = d_aff + cm, *add = d_aff + 2 * cm;

    // MeshSubdivideTables::build on the device: parent hash + child coords + child map
    s3dsp_hash* hash = nullptr;
    CALL(s3dsp_hash_build(ctx, static_cast<const int32_t*>(d_parents), np, 1, &hash, g_err, sizeof g_err));
    s3dsp_kmap* child = nullptr;
    CALL(s3dsp_subdivide(ctx, hash, d_child, &child, g_err, sizeof g_err));
    // GN1 + SiLU on the parents (sparse_group_norm, mesh_decoder_graph.cpp:16-30), bf16 for the tensor cores
    CALL(s3dsp_gn_stats(ctx, d_x, S3DSP_F32, np, cin, groups, d_part, g_err, sizeof g_err));
    CALL(s3dsp_gn_finalize(ctx, d_part, np, cin, groups, eps, static_cast<const float*>(d_gn1_w),
                           static_cast<const float*>(d_gn1_b), sub, mul, add, g_err, sizeof g_err));
    CALL(s3dsp_convert(ctx, d_x, S3DSP_F32, d_xb, S3DSP_BF16, np * cin, g_err, sizeof g_err));
    CALL(s3dsp_channel_affine(ctx, d_x, S3DSP_F32, np, cin, sub, mul, add, 1, d_h1, S3DSP_BF16, g_err, sizeof g_err));
    // conv1 over the children reading parent rows; GN2 partial sums from its epilogue
    CALL(s3dsp_conv(ctx, child, 27, P, d_h1, S3DSP_BF16, np, cin, 3, d_w1, static_cast<const float*>(d_conv1_b),
                    nullptr, 0, 0, d_y1, S3DSP_BF16, nc, cout, 0, nullptr, nullptr, nullptr, d_part, groups, g_err,
                    sizeof g_err));
    CALL(s3dsp_gn_finalize(ctx, d_part, nc, cout, groups, eps, static_cast<const float*>(d_gn2_w),
                           static_cast<const float*>(d_gn2_b), sub, mul, add, g_err, sizeof g_err));
    CALL(s3dsp_channel_affine(ctx, d_y1, S3DSP_BF16, nc, cout, sub, mul, add, 1, d_h2, S3DSP_BF16, g_err,
                              sizeof g_err));
    // 1x1 skip on the parents, then conv2 + the skip broadcast to the children
    CALL(s3dsp_conv(ctx, nullptr, 1, P, d_xb, S3DSP_BF16, np, cin, 0, d_ws, static_cast<const float*>(d_skip_b),
                    nullptr, 0, 0, d_skip, S3DSP_F32, np, cout, 0, nullptr, nullptr, nullptr, nullptr, 0, g_err,
                    sizeof g_err));
    CALL(s3dsp_conv(ctx, child, 27, P, d_h2, S3DSP_BF16, nc, cout, 0, d_w2, static_cast<const float*>(d_conv2_b),
                    d_skip, S3DSP_F32, 3, d_out, S3DSP_F32, nc, cout, 0, nullptr, nullptr, nullptr, nullptr, 0, g_err,
                    sizeof g_err));
    CALL(s3dsp_context_check(ctx, g_err, sizeof g_err));
    // read back (get_tensor_f32) and write the results
    std::vector<int32_t> h_child((size_t)(nc * 4));
    std::vector<float> h_out((size_t)(nc * cout));
    CALL(s3dsp_copy_to_host(ctx, h_child.data(), d_child, 16 * (uint64_t)nc, g_err, sizeof g_err));
    CALL(s3dsp_copy_to_host(ctx, h_out.data(), d_out, 4 * (uint64_t)(nc * cout), g_err, sizeof g_err));
    s3dsp_kmap_free(ctx, child);
    s3dsp_hash_free(ctx, hash);
    NEED(write_samt(dir + "/out_level_child_coords.samt", {nc, 4}, kGgmlI32, h_child.data(), 16 * (uint64_t)nc));
    NEED(write_samt(dir + "/out_level.samt", {nc, cout}, kGgmlF32, h_out.data(), 4 * (uint64_t)(nc * cout)));
    return 0;
}

// The config-2 residual block, BF16: conv3 -> GroupNorm(32) -> SiLU -> conv3
// -> + x over the submanifold map of the block's coordinates.
int run_block(s3dsp_context* ctx, Buffers& buf, const std::string& dir) {
    const uint32_t P = S3DSP_PREC_BF16;
    HostTensor coords, x, w1, b1, gamma, beta, w2, b2;
    const std::pair<const char*, HostTensor*> files[] = {
        {"block_coords", &coords}, {"block_x", &x},         {"block_w1", &w1}, {"block_b1", &b1},
        {"block_gamma", &gamma},   {"block_beta", &beta},   {"block_w2", &w2}, {"block_b2", &b2}};
    for (const auto& f : files)
        if (!read_samt(dir + "/" + f.first + ".samt", f.second)) return 1;
    const int64_t n = coords.dim(0), c = x.dim(1);
    const int32_t groups = 32;
    void* d_coords = buf.upload(coords);
    void* d_x = buf.upload(x);
    void* d_b1 = buf.upload(b1);
    void* d_b2 = buf.upload(b2);
    void* d_gamma = buf.upload(gamma);
    void* d_beta = buf.upload(beta);
    NEED(d_coords && d_x && d_b1 && d_b2 && d_gamma && d_beta);
    void* d_w1 = buf.pack(w1, S3DSP_LAYOUT_SLAT_ROW, 27, c, c, P);
    void* d_w2 = buf.pack(w2, S3DSP_LAYOUT_SLAT_ROW, 27, c, c, P);
    auto* d_part = static_cast<double*>(buf.get(8 * (uint64_t)s3dsp_gn_partials_count(n, c, groups)));
    auto* d_aff = static_cast<float*>(buf.get(4 * 3 * (uint64_t)c));
    void* d_xb = buf.get(2 * (uint64_t)(n * c));
    void* d_y1 = buf.get(2 * (uint64_t)(n * c));
    void* d_h = buf.get(2 * (uint64_t)(n * c));
    auto* d_out = static_cast<float*>(buf.get(4 * (uint64_t)(n * c)));
    NEED(d_w1 && d_w2 && d_part && d_aff && d_xb && d_y1 && d_h && d_out);
    s3dsp_hash* hash = nullptr;
    CALL(s3dsp_hash_build(ctx, static_cast<const int32_t*>(d_coords), n, 0, &hash, g_err, sizeof g_err));
    s3dsp_kmap* kmap = nullptr;
    CALL(s3dsp_kmap_build_subm3(ctx, hash, &kmap, g_err, sizeof g_err));
    CALL(s3dsp_convert(ctx, d_x, S3DSP_F32, d_xb, S3DSP_BF16, n * c, g_err, sizeof g_err));
    CALL(s3dsp_conv(ctx, kmap, 27, P, d_xb, S3DSP_BF16, n, c, 0, d_w1, static_cast<const float*>(d_b1), nullptr, 0, 0,
                    d_y1, S3DSP_BF16, n, c, 0, nullptr, nullptr, nullptr, d_part, groups, g_err, sizeof g_err));
    CALL(s3dsp_gn_finalize(ctx, d_part, n, c, groups, 1e-5f, static_cast<const float*>(d_gamma),
                           static_cast<const float*>(d_beta), d_aff, d_aff + c, d_aff + 2 * c, g_err, sizeof g_err));
    CALL(s3dsp_channel_affine(ctx, d_y1, S3DSP_BF16, n, c, d_aff, d_aff + c, d_aff + 2 * c, 1, d_h, S3DSP_BF16, g_err,
                              sizeof g_err));
    CALL(s3dsp_conv(ctx, kmap, 27, P, d_h, S3DSP_BF16, n, c, 0, d_w2, static_cast<const float*>(d_b2), d_x, S3DSP_F32,
                    0, d_out, S3DSP_F32, n, c, 0, nullptr, nullptr, nullptr, nullptr, 0, g_err, sizeof g_err));
    CALL(s3dsp_context_check(ctx, g_err, sizeof g_err));
    std::vector<float> h_out((size_t)(n * c));
    CALL(s3dsp_copy_to_host(ctx, h_out.data(), d_out, 4 * (uint64_t)(n * c), g_err, sizeof g_err));
    s3dsp_kmap_free(ctx, kmap);
    s3dsp_hash_free(ctx, hash);
    NEED(write_samt(dir + "/out_block.samt", {n, c}, kGgmlF32, h_out.data(), 4 * (uint64_t)(n * c)));
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc != 2) {
        std::fprintf(stderr, "usage: %s <dir>\n", argv[0]);
        return 2;
    }
    const std::string dir = argv[1];
    s3dsp_context* ctx = nullptr;
    // one context on device 0 and its own stream
    if (!ok(s3dsp_context_create(0, nullptr, S3DSP_CONTEXT_OWN_STREAM, &ctx, g_err, sizeof g_err),
            "s3dsp_context_create"))
        return 1;
    int rc;
    {
        Buffers buf;
        buf.ctx = ctx;
        rc = run_level(ctx, buf, dir);
        if (rc == 0) rc = run_block(ctx, buf, dir);
    }
    s3dsp_context_free(ctx);
    if (rc == 0) std::printf("capi_decode_level: ok\n");
    return rc;
}
