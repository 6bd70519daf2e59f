// TEST INFRASTRUCTURE ONLY — never linked into the product library.
//
// extern "C" wrappers around the reference's own host table builders so that
// Python tests (ctypes) can call them. The reference translation unit
// (src/objects_runtime/sparse_ops.cpp) is compiled unchanged, from where it
// lies in the reference tree, by oracle/Makefile; only this shim is ours.
//
// Wrapped entry points (reference file:line):
//   sam3d::SlatTables::build           src/objects_runtime/sparse_ops.cpp:49-173
//   sam3d::MeshSubdivideTables::build  src/objects_runtime/sparse_ops.cpp:272-404
//   sam3d::GsTables::build             src/objects_runtime/sparse_ops.cpp:182-270
//   sam3d::extract_object_mesh         src/objects_runtime/mesh_extractor.cpp:95-377
//     (compiled unchanged from mesh_extractor.cpp, with its generated
//     flexicubes_tables.hpp, which ref_flexicubes_tables copies out)
#include "flexicubes_tables.hpp"
#include "mesh_extractor.hpp"
#include "sparse_ops.hpp"

#include <string>
#include <vector>

#include <cstdint>
#include <cstring>

extern "C" {

// Runs SlatTables::build and copies every table out. The caller sizes the
// coarse outputs for the worst case (nc <= nf). Returns nc, or -1 when the
// reference builder returns false. `ape_channels` is forwarded unchanged
// (the APE table is not copied out; pass a small value such as 6).
int64_t ref_slat_tables(const int32_t* coords, int64_t nf, int32_t ape_channels,
                        int32_t* fine_to_coarse, int32_t* coarse_children,
                        float* coarse_inv_count, int32_t* conv_fine,
                        int32_t* conv_coarse) {
    sam3d::SlatTables t;
    if (!t.build(coords, nf, ape_channels)) return -1;
    std::memcpy(fine_to_coarse, t.fine_to_coarse.data(), t.fine_to_coarse.size() * 4);
    std::memcpy(coarse_children, t.coarse_children.data(), t.coarse_children.size() * 4);
    std::memcpy(coarse_inv_count, t.coarse_inv_count.data(), t.coarse_inv_count.size() * 4);
    std::memcpy(conv_fine, t.conv_fine.data(), t.conv_fine.size() * 4);
    std::memcpy(conv_coarse, t.conv_coarse.data(), t.conv_coarse.size() * 4);
    return t.nc;
}

// Runs MeshSubdivideTables::build. Outputs are [8*count, 4] child coords and
// [8*count, 27] child-major neighbours (-1 = missing). Returns 1 on success,
// 0 when the reference builder returns false.
int32_t ref_mesh_subdivide(const int32_t* parent_coords, int64_t count,
                           int32_t* child_coords, int32_t* neighbors) {
    sam3d::MeshSubdivideTables t;
    if (!t.build(parent_coords, count)) return 0;
    std::memcpy(child_coords, t.child_coords.data(), t.child_coords.size() * 4);
    std::memcpy(neighbors, t.neighbors.data(), t.neighbors.size() * 4);
    return 1;
}

// Runs GsTables::build and copies out shift `si`'s tables (bkt_idx, bwd_idx,
// buckets as {len, off, n_win} triples) and, when ape is not NULL, the
// (n, 768) position embedding. Returns the bucket count, or -1 when the
// reference builder returns false.
int64_t ref_gs_tables(const int32_t* coords, int64_t n, int32_t si, int32_t* bkt_idx, int32_t* bwd_idx,
                      int32_t* buckets, float* ape) {
    sam3d::GsTables t;
    if (!t.build(coords, n)) return -1;
    const sam3d::GsWindowTables& w = t.shifts[si];
    std::memcpy(bkt_idx, w.bkt_idx.data(), w.bkt_idx.size() * 4);
    std::memcpy(bwd_idx, w.bwd_idx.data(), w.bwd_idx.size() * 4);
    for (size_t k = 0; k < w.buckets.size(); ++k) {
        buckets[3 * k + 0] = w.buckets[k].len;
        buckets[3 * k + 1] = w.buckets[k].off;
        buckets[3 * k + 2] = w.buckets[k].n_win;
    }
    if (ape) std::memcpy(ape, t.ape.data(), t.ape.size() * 4);
    return (int64_t)w.buckets.size();
}

// Copies the reference's DMC tables: dmc [256][4][7], num_dual [256],
// check [256][5].
void ref_flexicubes_tables(int8_t* dmc, int8_t* num_dual, int16_t* check) {
    namespace t = sam3d::flexicubes_tables;
    std::memcpy(dmc, t::dmc, sizeof t::dmc);
    std::memcpy(num_dual, t::num_dual, sizeof t::num_dual);
    std::memcpy(check, t::check, sizeof t::check);
}

static sam3d::ObjectMesh g_mesh;
static sam3d::MeshExtractionTaps g_taps;

// Runs extract_object_mesh with taps. Returns 0, or -1 when the reference
// returns false (the message goes to `error`). counts: {dual vertices,
// triangles, surface cubes, surface edges}.
int32_t ref_flexicubes(const float* raw, const int32_t* coords, int64_t n, int64_t* counts, char* error,
                       int64_t error_capacity) {
    std::string msg;
    if (!sam3d::extract_object_mesh(raw, coords, n, g_mesh, &g_taps, &msg)) {
        if (error && error_capacity > 0) {
            std::strncpy(error, msg.c_str(), (size_t)error_capacity - 1);
            error[error_capacity - 1] = '\0';
        }
        return -1;
    }
    counts[0] = (int64_t)g_mesh.vertices.size() / 3;
    counts[1] = (int64_t)g_mesh.faces.size() / 3;
    counts[2] = (int64_t)g_taps.surface_cube_indices.size();
    counts[3] = (int64_t)g_taps.surface_edges.size() / 2;
    return 0;
}

// Copies the last ref_flexicubes result; any pointer may be NULL.
void ref_flexicubes_fetch(float* vertices, float* attrs, int32_t* faces, int32_t* surface, int32_t* cases,
                          int32_t* edges) {
    const auto put = [](auto* dst, const auto& v) {
        if (dst && !v.empty()) std::memcpy(dst, v.data(), v.size() * sizeof(v[0]));
    };
    put(vertices, g_mesh.vertices);
    put(attrs, g_mesh.vertex_attributes);
    put(faces, g_mesh.faces);
    put(surface, g_taps.surface_cube_indices);
    put(cases, g_taps.case_ids);
    put(edges, g_taps.surface_edges);
}

}  // extern "C"
