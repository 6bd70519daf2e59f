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
#include "sparse_ops.hpp"

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

}  // extern "C"
