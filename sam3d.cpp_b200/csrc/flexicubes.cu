// FlexiCubes extraction at resolution 256 on the device: extract_object_mesh
// (src/objects_runtime/mesh_extractor.cpp:95-377), SparseFeatures2Mesh
// followed by inference-mode FlexiCubes.
//
// Layout: dense grids over the 256^3 cubes and 257^3 vertices (x-major, z
// fastest) instead of hash maps: cube -> input row, vertex -> SDF, vertex ->
// attribute slot, cube -> occupancy byte, cube -> surface index.
//
//  1. cube_row[cube] = lowest input row (atomicMin); per-row checks of batch,
//     range and duplicates record the first offending row of each kind.
//  2. A warp per (x, y) row of 257 vertices writes every vertex's SDF (1 where
//     no cube holds it) and attribute slot: a vertex's (<= 8) holding cubes
//     are read coalesced along z, sorted by row in registers (a 19-comparator
//     network on row << 3 | corner) and summed in that order -- the
//     reference's accumulation order, so the means are bit-identical to the
//     host's. Slot = lowest row * 8 + its corner.
//  3. A warp per (x, y) row of 256 cubes computes the occupancy bytes and
//     counts the surface cubes (ballot); a warp per (x, y) row of 257
//     vertices counts the sign-changing edges starting there (the -y, +z, +x
//     edge of vertex u, which is the reference's (first, second) key order)
//     and the quads among them (edges with four cubes in range), split by
//     orientation. One scan per row list gives every row its output offsets,
//     so both lists come out in the reference's order without a sort.
//  4. Per surface cube: the ambiguous-case check against the neighbour's raw
//     case, then the dual vertices, numbered by (dual count, surface index,
//     local index) through an int4 scan of one-hot dual counts.
//  5. The edge pass records each quad (a surface edge with four cubes in the
//     grid) at its slot, flipped quads first; a thread per quad then joins
//     the four cubes' dual vertices in dense cube order and writes the two
//     triangles, split by the gamma products.
//
// Arithmetic follows the reference's order with no contraction (explicit
// _rn intrinsics); tanhf / expf are CUDA's, so positions and attributes match
// the host to a few ulps while the topology (surface cubes, cases, edges,
// faces) is identical.
#include "s3dsp_internal.h"

#include <cub/cub.cuh>

#include <climits>

using namespace s3dsp;

struct s3dsp_fc_tables {
    int8_t* dmc = nullptr;       // [256][4][7]
    int8_t* num_dual = nullptr;  // [256]
    int16_t* check = nullptr;    // [256][5]
    void* base = nullptr;
};

struct s3dsp_mesh {
    int64_t n_vertices = 0, n_faces = 0, n_surface = 0, n_edges = 0;
    float* vertices = nullptr;  // [V, 3]
    float* attrs = nullptr;     // [V, 6]
    int32_t* faces = nullptr;   // [F, 3]
    int32_t* surface = nullptr; // [S]
    int32_t* cases = nullptr;   // [S]
    int32_t* edges = nullptr;   // [E, 2]
};

namespace {

constexpr int R = 256;
constexpr int RV = 257;
constexpr int RAW = 101;
constexpr int32_t kNoRow = 0x7F7F7F7F;  // memset(0x7F) fill: above every row index
constexpr int64_t kCubes = (int64_t)R * R * R;
constexpr int64_t kVerts = (int64_t)RV * RV * RV;

// corner k = (k & 1, k >> 1 & 1, k >> 2 & 1); edge e runs kEdgeA[e] -> kEdgeB[e]
__constant__ int8_t kEdgeA[12] = {0, 1, 4, 0, 2, 3, 6, 2, 2, 3, 7, 6};
__constant__ int8_t kEdgeB[12] = {1, 5, 5, 4, 3, 7, 7, 6, 0, 1, 5, 4};

__device__ __forceinline__ int32_t vid(int x, int y, int z) { return (x * RV + y) * RV + z; }
__device__ __forceinline__ int32_t cid(int x, int y, int z) { return (x * R + y) * R + z; }
__device__ __forceinline__ bool in_grid(int x, int y, int z) {
    return (unsigned)x < (unsigned)R && (unsigned)y < (unsigned)R && (unsigned)z < (unsigned)R;
}

// error kinds, in the reference's per-row check order
enum { kErrBatch = 0, kErrRange = 1, kErrDup = 2 };

struct Int4Add {
    __host__ __device__ int4 operator()(const int4& a, const int4& b) const {
        return make_int4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
    }
};

__global__ void fc_scatter_kernel(const int4* __restrict__ coords, int64_t n, int32_t* __restrict__ cube_row,
                                  int32_t* __restrict__ err_row) {
    pdl_wait();
    pdl_trigger();
    const int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (r >= n) return;
    const int4 c = coords[r];
    if (c.x != 0) {
        atomicMin(err_row + kErrBatch, (int32_t)r);
        return;
    }
    if (!in_grid(c.y, c.z, c.w)) {
        atomicMin(err_row + kErrRange, (int32_t)r);
        return;
    }
    atomicMin(cube_row + cid(c.y, c.z, c.w), (int32_t)r);
}

// A row whose cube already holds a lower row is the reference's duplicate.
__global__ void fc_dup_kernel(const int4* __restrict__ coords, int64_t n, const int32_t* __restrict__ cube_row,
                              int32_t* __restrict__ err_row) {
    pdl_wait();
    pdl_trigger();
    const int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (r >= n) return;
    const int4 c = coords[r];
    if (c.x != 0 || !in_grid(c.y, c.z, c.w)) return;
    if (cube_row[cid(c.y, c.z, c.w)] != (int32_t)r) atomicMin(err_row + kErrDup, (int32_t)r);
}

__device__ __forceinline__ void cswap(int32_t& a, int32_t& b) {
    const int32_t lo = min(a, b), hi = max(a, b);
    a = lo;
    b = hi;
}

constexpr int kVChunks = (RV + 31) / 32;  // 32-vertex chunks per (x, y) row

// Warp per 32 vertices of an (x, y) row (lane = z offset). Vertex (x, y, z)
// is corner k of cube (x - (k & 1), y - (k >> 1 & 1), z - (k >> 2 & 1)).
__global__ void fc_vertex_kernel(const float* __restrict__ raw, const int32_t* __restrict__ cube_row,
                                 float* __restrict__ sdf, int32_t* __restrict__ vslot, float* __restrict__ vattr) {
    pdl_wait();
    pdl_trigger();
    const int w = (int)((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (w >= RV * RV * kVChunks) return;
    const int row = w / kVChunks;
    const int x = row / RV, y = row % RV;
    const int z = (w % kVChunks) * 32 + lane;
    if (z < RV) {
        int32_t rk[8];  // row << 3 | corner, INT_MAX when the cube is absent
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int cx = x - (k & 1), cy = y - (k >> 1 & 1), cz = z - (k >> 2 & 1);
            const int32_t r = in_grid(cx, cy, cz) ? cube_row[cid(cx, cy, cz)] : kNoRow;
            rk[k] = r == kNoRow ? INT_MAX : (r << 3 | k);
        }
        const int32_t v = vid(x, y, z);
        if ((rk[0] & rk[1] & rk[2] & rk[3] & rk[4] & rk[5] & rk[6] & rk[7]) == INT_MAX) {
            sdf[v] = 1.0f;
            vslot[v] = -1;
            return;
        }
        cswap(rk[0], rk[2]), cswap(rk[1], rk[3]), cswap(rk[4], rk[6]), cswap(rk[5], rk[7]);
        cswap(rk[0], rk[4]), cswap(rk[1], rk[5]), cswap(rk[2], rk[6]), cswap(rk[3], rk[7]);
        cswap(rk[0], rk[1]), cswap(rk[2], rk[3]), cswap(rk[4], rk[5]), cswap(rk[6], rk[7]);
        cswap(rk[2], rk[4]), cswap(rk[3], rk[5]);
        cswap(rk[1], rk[4]), cswap(rk[3], rk[6]);
        cswap(rk[1], rk[2]), cswap(rk[3], rk[4]), cswap(rk[5], rk[6]);
        float sum[10];
#pragma unroll
        for (int ch = 0; ch < 10; ++ch) sum[ch] = 0.0f;
        // Absent cubes (sorted last) read the first cube's row and add +0,
        // which leaves a sum that starts at +0 unchanged, so every load can be
        // in flight at once.
        int m = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const bool ok = rk[i] != INT_MAX;
            m += ok;
            const int32_t e = ok ? rk[i] : rk[0];
            const float* f = raw + (int64_t)(e >> 3) * RAW;
            const int k = e & 7;
            const float t0 = __fsub_rn(__ldg(f + k), 1.0f / R);
            sum[0] = __fadd_rn(sum[0], ok ? t0 : 0.0f);
#pragma unroll
            for (int a = 0; a < 3; ++a) {
                const float t = __ldg(f + 8 + 3 * k + a);
                sum[1 + a] = __fadd_rn(sum[1 + a], ok ? t : 0.0f);
            }
#pragma unroll
            for (int ch = 0; ch < 6; ++ch) {
                const float t = __ldg(f + 53 + 6 * k + ch);
                sum[4 + ch] = __fadd_rn(sum[4 + ch], ok ? t : 0.0f);
            }
        }
        const float fm = (float)m;
        const int32_t slot = rk[0];  // lowest row * 8 + its corner
        float* o = vattr + (int64_t)slot * 9;
        const int p[3] = {x, y, z};
#pragma unroll
        for (int a = 0; a < 3; ++a) {
            const float mean = __fdiv_rn(sum[1 + a], fm);
            o[a] = __fadd_rn(__fsub_rn(__fdiv_rn((float)p[a], (float)R), 0.5f), __fmul_rn(1.0f / (R * 2.0f), tanhf(mean)));
        }
#pragma unroll
        for (int ch = 0; ch < 6; ++ch) {
            const float mean = __fdiv_rn(sum[4 + ch], fm);
            o[3 + ch] = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-mean)));
        }
        sdf[v] = __fdiv_rn(sum[0], fm);
        vslot[v] = slot;
    }
}

// Warp per (x, y) row of 256 cubes: occupancy bytes + surface count.
__global__ void fc_surface_count_kernel(const float* __restrict__ sdf, uint8_t* __restrict__ occ,
                                        int32_t* __restrict__ row_count) {
    pdl_wait();
    pdl_trigger();
    const int row = (int)((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= R * R) return;
    const int x = row >> 8, y = row & 255;
    const float* s00 = sdf + vid(x, y, 0);
    const float* s10 = sdf + vid(x + 1, y, 0);
    const float* s01 = sdf + vid(x, y + 1, 0);
    const float* s11 = sdf + vid(x + 1, y + 1, 0);
    int total = 0;
#pragma unroll 2
    for (int j = 0; j < R / 32; ++j) {
        const int z = lane + 32 * j;
        const unsigned bits = (unsigned)(s00[z] < 0.0f) | (unsigned)(s10[z] < 0.0f) << 1 |
                              (unsigned)(s01[z] < 0.0f) << 2 | (unsigned)(s11[z] < 0.0f) << 3 |
                              (unsigned)(s00[z + 1] < 0.0f) << 4 | (unsigned)(s10[z + 1] < 0.0f) << 5 |
                              (unsigned)(s01[z + 1] < 0.0f) << 6 | (unsigned)(s11[z + 1] < 0.0f) << 7;
        occ[cid(x, y, z)] = (uint8_t)bits;
        total += __popc(__ballot_sync(0xffffffffu, bits != 0u && bits != 255u));
    }
    if (lane == 0) row_count[row] = total;
}

// The three edges that start at vertex (x, y, z) in key order (-y, +z, +x):
// bit d of `edges` = edge d changes sign; bit d of `quads` = it also has four
// cubes inside the grid.
__device__ __forceinline__ void vertex_edges(const float* __restrict__ sdf, int x, int y, int z, unsigned& edges,
                                             unsigned& quads, bool& flip) {
    const int32_t u = vid(x, y, z);
    const float s = sdf[u];
    const bool neg = s < 0.0f;
    flip = s > 0.0f;
    edges = 0;
    if (y >= 1 && neg != (sdf[u - RV] < 0.0f)) edges |= 1u;
    if (z < R && neg != (sdf[u + 1] < 0.0f)) edges |= 2u;
    if (x < R && neg != (sdf[u + RV * RV] < 0.0f)) edges |= 4u;
    const bool ix = x >= 1 && x < R, iy = y >= 1 && y < R, iz = z >= 1 && z < R;
    quads = edges & ((ix && iz ? 1u : 0u) | (ix && iy ? 2u : 0u) | (iy && iz ? 4u : 0u));
}

// Warp per (x, y) row of 257 vertices: {edges, flipped quads, other quads}.
__global__ void fc_edge_count_kernel(const float* __restrict__ sdf, int4* __restrict__ row_count) {
    pdl_wait();
    pdl_trigger();
    const int row = (int)((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= RV * RV) return;
    const int x = row / RV, y = row % RV;
    int ne = 0, nqf = 0, nqn = 0;
    for (int z = lane; z < RV; z += 32) {
        unsigned e, q;
        bool flip;
        vertex_edges(sdf, x, y, z, e, q, flip);
        ne += __popc(e);
        (flip ? nqf : nqn) += __popc(q);
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
        ne += __shfl_xor_sync(0xffffffffu, ne, d);
        nqf += __shfl_xor_sync(0xffffffffu, nqf, d);
        nqn += __shfl_xor_sync(0xffffffffu, nqn, d);
    }
    if (lane == 0) row_count[row] = make_int4(ne, nqf, nqn, 0);
}

// totals[0] = surface cubes, [1..3] = edges, flipped quads, other quads,
// [4..6] = first bad row per error kind (INT_MAX when none).
__global__ void fc_totals_kernel(const int32_t* __restrict__ srow_count, const int32_t* __restrict__ srow_off,
                                 const int4* __restrict__ erow_count, const int4* __restrict__ erow_off,
                                 const int32_t* __restrict__ err_row, int64_t* __restrict__ totals) {
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    totals[0] = (int64_t)srow_off[R * R - 1] + srow_count[R * R - 1];
    const int4 a = erow_off[RV * RV - 1], b = erow_count[RV * RV - 1];
    totals[1] = (int64_t)a.x + b.x;
    totals[2] = (int64_t)a.y + b.y;
    totals[3] = (int64_t)a.z + b.z;
    for (int k = 0; k < 3; ++k) totals[4 + k] = err_row[k];
}

// Warp per (x, y) row of cubes: the surface list in dense order.
__global__ void fc_surface_write_kernel(const uint8_t* __restrict__ occ, const int32_t* __restrict__ row_off,
                                        int32_t* __restrict__ surf, int32_t* __restrict__ sidx) {
    pdl_wait();
    pdl_trigger();
    const int row = (int)((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= R * R) return;
    int32_t off = row_off[row];
    const int32_t c0 = row * R;  // cid(x, y, 0)
    for (int j = 0; j < R / 32; ++j) {
        const int32_t c = c0 + lane + 32 * j;
        const unsigned b = occ[c];
        const bool f = b != 0u && b != 255u;
        const unsigned mask = __ballot_sync(0xffffffffu, f);
        if (f) {
            const int32_t pos = off + __popc(mask & ((1u << lane) - 1u));
            surf[pos] = c;
            sidx[c] = pos;
        }
        off += __popc(mask);
    }
}

// Per surface cube: resolved case (ambiguity check against the face
// neighbour's raw case) and a one-hot of its dual-vertex count.
__global__ void fc_case_kernel(const int32_t* __restrict__ surf, int64_t ns, const uint8_t* __restrict__ occ,
                               const int8_t* __restrict__ num_dual, const int16_t* __restrict__ check,
                               int32_t* __restrict__ cases, int4* __restrict__ onehot) {
    pdl_wait();
    pdl_trigger();
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= ns) return;
    const int32_t c = surf[i];
    int cs = occ[c];
    const int16_t* ck = check + 5 * cs;
    if (ck[0] == 1) {
        const int nx = c / (R * R) + ck[1], ny = c / R % R + ck[2], nz = c % R + ck[3];
        if (in_grid(nx, ny, nz)) {
            const int nb = occ[cid(nx, ny, nz)];
            if (nb != 0 && nb != 255 && check[5 * nb] == 1) cs = ck[4];
        }
    }
    cases[i] = cs;
    const int nd = num_dual[cs];
    onehot[i] = make_int4(nd == 1, nd == 2, nd == 3, nd == 4);
}

__device__ __forceinline__ int pick(const int4& v, int k) { return k == 1 ? v.x : k == 2 ? v.y : k == 3 ? v.z : v.w; }

__device__ __forceinline__ void vertex_attr(int32_t v, const int32_t* __restrict__ vslot,
                                            const float* __restrict__ vattr, float out[9]) {
    const int32_t s = vslot[v];
    if (s >= 0) {
#pragma unroll
        for (int k = 0; k < 9; ++k) out[k] = vattr[(int64_t)s * 9 + k];
        return;
    }
    const int p[3] = {v / (RV * RV), v / RV % RV, v % RV};
#pragma unroll
    for (int a = 0; a < 3; ++a) out[a] = __fsub_rn(__fdiv_rn((float)p[a], (float)R), 0.5f);
#pragma unroll
    for (int ch = 0; ch < 6; ++ch) out[3 + ch] = 0.5f;
}

// Per surface cube: its dual vertices (id = base[nd] + rank * nd + j) and the
// cube's 12-entry edge -> dual vertex map (0 where no dual vertex lists the
// edge, as the reference initialises it).
__global__ void fc_dual_kernel(const int32_t* __restrict__ surf, int64_t ns, const int32_t* __restrict__ cases,
                               const int4* __restrict__ onehot, const int4* __restrict__ rank,
                               const int32_t* __restrict__ cube_row, const float* __restrict__ raw,
                               const float* __restrict__ sdf, const int32_t* __restrict__ vslot,
                               const float* __restrict__ vattr, const int8_t* __restrict__ dmc,
                               const int8_t* __restrict__ num_dual, float* __restrict__ out_v,
                               float* __restrict__ out_a, float* __restrict__ dual_gamma,
                               int32_t* __restrict__ dmap, int64_t* __restrict__ n_dual) {
    pdl_wait();
    pdl_trigger();
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    // dual vertices of each count: totals = last exclusive rank + last one-hot
    const int4 tot = Int4Add()(rank[ns - 1], onehot[ns - 1]);
    int64_t base[5];
    base[0] = 0;
    base[1] = 0;
    base[2] = base[1] + (int64_t)tot.x;
    base[3] = base[2] + (int64_t)tot.y * 2;
    base[4] = base[3] + (int64_t)tot.z * 3;
    if (i == 0) *n_dual = base[4] + (int64_t)tot.w * 4;
    if (i >= ns) return;
    const int32_t c = surf[i];
    const int cs = cases[i];
    const int nd = num_dual[cs];
    int32_t dm[12];
#pragma unroll
    for (int e = 0; e < 12; ++e) dm[e] = 0;
    if (nd > 0) {
        const int cx = c / (R * R), cy = c / R % R, cz = c % R;
        int32_t vtx[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) vtx[k] = vid(cx + (k & 1), cy + (k >> 1 & 1), cz + (k >> 2 & 1));
        const int32_t row = cube_row[c];
        const float* w = row == kNoRow ? nullptr : raw + (int64_t)row * RAW + 32;
        float alpha[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) alpha[k] = __fadd_rn(__fmul_rn(tanhf(w ? __ldg(w + 12 + k) : 0.0f), 0.99f), 1.0f);
        const float g20 = w ? __ldg(w + 20) : 0.0f;
        const float gamma = __fadd_rn(__fmul_rn(__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g20))), 0.99f), 0.005f);
        const int64_t first = base[nd] + (int64_t)pick(rank[i], nd) * nd;
        for (int j = 0; j < nd; ++j) {
            const int64_t id = first + j;
            float pos[3] = {0.0f, 0.0f, 0.0f}, col[6] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f}, beta_sum = 0.0f;
            for (int t = 0; t < 7; ++t) {
                const int e = dmc[(cs * 4 + j) * 7 + t];
                if (e < 0) continue;
                const int ka = kEdgeA[e], kb = kEdgeB[e];
                const float wa = __fmul_rn(sdf[vtx[ka]], alpha[ka]);
                const float wb = __fmul_rn(sdf[vtx[kb]], alpha[kb]);
                const float den = __fsub_rn(wb, wa);
                float va[9], vb[9];
                vertex_attr(vtx[ka], vslot, vattr, va);
                vertex_attr(vtx[kb], vslot, vattr, vb);
                const float beta = __fadd_rn(__fmul_rn(tanhf(w ? __ldg(w + e) : 0.0f), 0.99f), 1.0f);
                beta_sum = __fadd_rn(beta_sum, beta);
#pragma unroll
                for (int a = 0; a < 3; ++a)
                    pos[a] = __fadd_rn(pos[a], __fmul_rn(__fdiv_rn(__fsub_rn(__fmul_rn(va[a], wb), __fmul_rn(vb[a], wa)), den), beta));
#pragma unroll
                for (int ch = 0; ch < 6; ++ch)
                    col[ch] = __fadd_rn(col[ch], __fmul_rn(__fdiv_rn(__fsub_rn(__fmul_rn(va[3 + ch], wb), __fmul_rn(vb[3 + ch], wa)), den), beta));
                dm[e] = (int32_t)id;
            }
#pragma unroll
            for (int a = 0; a < 3; ++a) out_v[id * 3 + a] = __fdiv_rn(pos[a], beta_sum);
#pragma unroll
            for (int ch = 0; ch < 6; ++ch) out_a[id * 6 + ch] = __fdiv_rn(col[ch], beta_sum);
            dual_gamma[id] = gamma;
        }
    }
    int4* d4 = reinterpret_cast<int4*>(dmap + i * 12);
    d4[0] = make_int4(dm[0], dm[1], dm[2], dm[3]);
    d4[1] = make_int4(dm[4], dm[5], dm[6], dm[7]);
    d4[2] = make_int4(dm[8], dm[9], dm[10], dm[11]);
}

// The quad of the edge u -> v (direction d: 0 = -y, 1 = +z, 2 = +x) over its
// four cubes in dense order, written as two triangles.
__device__ void emit_quad(int x, int y, int z, int d, int32_t u, int32_t v, bool flip,
                          const int32_t* __restrict__ sidx, const int32_t* __restrict__ dmap,
                          const float* __restrict__ dual_gamma, int32_t* __restrict__ tri) {
    int32_t cubes[4];
    int m = 0;
#pragma unroll
    for (int d0 = 1; d0 >= 0; --d0)
#pragma unroll
        for (int d1 = 1; d1 >= 0; --d1) {
            int cx = x, cy = y, cz = z;
            if (d == 2) cy -= d0, cz -= d1;
            else if (d == 1) cx -= d0, cy -= d1;
            else cx -= d0, cy -= 1, cz -= d1;
            cubes[m++] = cid(cx, cy, cz);
        }
    // (d0, d1) = (1,1), (1,0), (0,1), (0,0) is ascending dense order for all
    // three directions; the network below keeps the order explicit.
#pragma unroll
    for (int a = 0; a < 3; ++a)
#pragma unroll
        for (int b = 0; b < 3 - a; ++b)
            if (cubes[b] > cubes[b + 1]) {
                const int32_t t = cubes[b];
                cubes[b] = cubes[b + 1];
                cubes[b + 1] = t;
            }
    int32_t q[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int32_t c = cubes[j];
        const int cx = c / (R * R), cy = c / R % R, cz = c % R;
        int e = 0;
        for (; e < 11; ++e) {
            const int ka = kEdgeA[e], kb = kEdgeB[e];
            if (vid(cx + (ka & 1), cy + (ka >> 1 & 1), cz + (ka >> 2 & 1)) == u &&
                vid(cx + (kb & 1), cy + (kb >> 1 & 1), cz + (kb >> 2 & 1)) == v)
                break;
        }
        q[j] = dmap[(int64_t)sidx[c] * 12 + e];
    }
    const int32_t o0 = flip ? q[0] : q[2], o1 = flip ? q[1] : q[3], o2 = flip ? q[3] : q[1], o3 = flip ? q[2] : q[0];
    const bool split1 = __fmul_rn(dual_gamma[o0], dual_gamma[o2]) > __fmul_rn(dual_gamma[o1], dual_gamma[o3]);
    if (split1) {
        tri[0] = o0, tri[1] = o1, tri[2] = o2, tri[3] = o0, tri[4] = o2, tri[5] = o3;
    } else {
        tri[0] = o0, tri[1] = o1, tri[2] = o3, tri[3] = o3, tri[4] = o1, tri[5] = o2;
    }
}

// Warp per (x, y) row of vertices: writes the surface edges in key order and
// a record {u, direction, flip} for each quad at its slot (flipped first).
__global__ void fc_edge_write_kernel(const float* __restrict__ sdf, const int4* __restrict__ row_off,
                                     const int64_t* __restrict__ totals, int32_t* __restrict__ edges,
                                     int32_t* __restrict__ quads) {
    pdl_wait();
    pdl_trigger();
    const int row = (int)((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= RV * RV) return;
    const int x = row / RV, y = row % RV;
    const int64_t flipped_total = totals[2];
    int4 off = row_off[row];
    for (int z0 = 0; z0 < RV; z0 += 32) {
        const int z = z0 + lane;
        unsigned e = 0, q = 0;
        bool flip = false;
        if (z < RV) vertex_edges(sdf, x, y, z, e, q, flip);
        // one warp scan over packed counts: edges | flipped quads << 10 | other quads << 20
        const int mine = __popc(e) | (flip ? __popc(q) << 10 : __popc(q) << 20);
        int incl = mine;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl, d);
            if (lane >= d) incl += t;
        }
        const int excl = incl - mine;
        if (e) {
            const int32_t u = vid(x, y, z);
            const int32_t second[3] = {u - RV, u + 1, u + RV * RV};
            int32_t ep = off.x + (excl & 1023);
            int64_t qp = flip ? off.y + (excl >> 10 & 1023) : flipped_total + off.z + (excl >> 20 & 1023);
#pragma unroll
            for (int d = 0; d < 3; ++d) {
                if (!(e >> d & 1u)) continue;
                edges[(int64_t)ep * 2] = u;
                edges[(int64_t)ep * 2 + 1] = second[d];
                ++ep;
                if (q >> d & 1u) quads[qp++] = u | d << 25 | (int32_t)flip << 27;
            }
        }
        const int total = __shfl_sync(0xffffffffu, incl, 31);
        off.x += total & 1023;
        off.y += total >> 10 & 1023;
        off.z += total >> 20 & 1023;
    }
}

// Thread per quad record (u < 2^25 vertices, direction in bits 25-26, flip in bit 27).
__global__ void fc_quad_kernel(const int32_t* __restrict__ quads, int64_t nq, const int32_t* __restrict__ sidx,
                               const int32_t* __restrict__ dmap, const float* __restrict__ dual_gamma,
                               int32_t* __restrict__ faces) {
    pdl_wait();
    pdl_trigger();
    const int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (q >= nq) return;
    const int32_t rec = quads[q];
    const int32_t u = rec & ((1 << 25) - 1);
    const int d = rec >> 25 & 3;
    const bool flip = rec >> 27 & 1;
    const int x = u / (RV * RV), y = u / RV % RV, z = u % RV;
    const int32_t v = d == 0 ? u - RV : d == 1 ? u + 1 : u + RV * RV;
    emit_quad(x, y, z, d, u, v, flip, sidx, dmap, dual_gamma, faces + q * 6);
}

int grid_for(int64_t n, int threads) {
    const int64_t g = (n + threads - 1) / threads;
    return (int)(g < 1 ? 1 : g);
}

struct Scratch {
    cudaStream_t s;
    void* ptrs[32];
    int count = 0;
    explicit Scratch(cudaStream_t st) : s(st) {}
    ~Scratch() {
        for (int i = 0; i < count; ++i) cudaFreeAsync(ptrs[i], s);
    }
    template <typename T>
    cudaError_t get(T** p, size_t bytes) {
        void* q = nullptr;
        const cudaError_t e = count < 32 ? s3dsp::malloc_async(&q, bytes > 0 ? bytes : 16, s) : cudaErrorMemoryAllocation;
        if (e == cudaSuccess) ptrs[count++] = q;
        *p = static_cast<T*>(q);
        return e;
    }
};

void mesh_release(s3dsp_mesh* m, cudaStream_t st) {
    if (!m) return;
    void* bufs[6] = {m->vertices, m->attrs, m->faces, m->surface, m->cases, m->edges};
    for (void* b : bufs)
        if (b) cudaFreeAsync(b, st);
    delete m;
}

}  // namespace

extern "C" S3DSP_API s3d_status s3dsp_flexicubes_tables_create(s3dsp_context* ctx, const int8_t* h_dmc,
                                                               const int8_t* h_num_dual, const int16_t* h_check,
                                                               s3dsp_fc_tables** out, char* error,
                                                               uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !h_dmc || !h_num_dual || !h_check || !out)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    *out = nullptr;
    for (int c = 0; c < 256; ++c) {
        if (h_num_dual[c] < 0 || h_num_dual[c] > 4)
            return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "num_dual[%d] = %d outside [0, 4]", c, h_num_dual[c]);
        for (int k = 0; k < 28; ++k)
            if (h_dmc[c * 28 + k] < -1 || h_dmc[c * 28 + k] > 11)
                return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "dmc[%d] entry %d outside [-1, 11]", c, k);
        const int16_t* ck = h_check + 5 * c;
        if (ck[0] == 1 && (ck[4] < 0 || ck[4] > 255))
            return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "check[%d] replacement case %d", c, ck[4]);
    }
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    constexpr size_t kDmc = 256 * 28, kNd = 256, kCk = 256 * 5 * 2;
    auto* t = new (std::nothrow) s3dsp_fc_tables;
    if (!t) return fail(error, error_capacity, S3D_OUT_OF_MEMORY, "host allocation");
    cudaError_t e = cudaMalloc(&t->base, kDmc + kNd + kCk);
    if (e == cudaSuccess) {
        t->check = static_cast<int16_t*>(t->base);
        t->dmc = static_cast<int8_t*>(t->base) + kCk;
        t->num_dual = t->dmc + kDmc;
        e = cudaMemcpy(t->check, h_check, kCk, cudaMemcpyHostToDevice);
    }
    if (e == cudaSuccess) e = cudaMemcpy(t->dmc, h_dmc, kDmc, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(t->num_dual, h_num_dual, kNd, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        if (t->base) cudaFree(t->base);
        delete t;
        return cuda_fail(error, error_capacity, e, "flexicubes tables");
    }
    *out = t;
    return S3D_OK;
}

extern "C" S3DSP_API void s3dsp_flexicubes_tables_free(s3dsp_context* ctx, s3dsp_fc_tables* tables) {
    if (!tables) return;
    if (ctx) cudaSetDevice(ctx->device);
    if (tables->base) cudaFree(tables->base);
    delete tables;
}

extern "C" S3DSP_API s3d_status s3dsp_flexicubes_extract(s3dsp_context* ctx, const s3dsp_fc_tables* tables,
                                                         const float* d_raw, const int32_t* d_coords, int64_t n,
                                                         s3dsp_mesh** out, char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (out) *out = nullptr;
    if (!ctx || !tables || !out) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    if (!d_raw || !d_coords || n <= 0 || n > INT32_MAX)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "invalid mesh decoder tensor");
    if (n > kCubes)  // more rows than cubes: some coordinate repeats or lies outside
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "duplicate mesh cube coordinate");
    if ((uintptr_t)d_coords & 15)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "d_coords must be 16-byte aligned");
    if ((uintptr_t)d_raw & 3) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "d_raw must be 4-byte aligned");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    cudaStream_t st = ctx->stream;
    const int4* coords = reinterpret_cast<const int4*>(d_coords);
    Scratch sc(st);
    int32_t *cube_row, *vslot, *sidx, *err_row, *srow_count, *srow_off;
    float *sdf, *vattr;
    uint8_t* occ;
    int4 *erow_count, *erow_off;
    int64_t* totals;
    cudaError_t e = sc.get(&cube_row, 4 * kCubes);
    if (e == cudaSuccess) e = sc.get(&sdf, 4 * kVerts);
    if (e == cudaSuccess) e = sc.get(&vslot, 4 * kVerts);
    if (e == cudaSuccess) e = sc.get(&vattr, 36 * 8 * (size_t)n);
    if (e == cudaSuccess) e = sc.get(&occ, kCubes);
    if (e == cudaSuccess) e = sc.get(&sidx, 4 * kCubes);
    if (e == cudaSuccess) e = sc.get(&err_row, 16);
    if (e == cudaSuccess) e = sc.get(&srow_count, 4 * R * R);
    if (e == cudaSuccess) e = sc.get(&srow_off, 4 * R * R);
    if (e == cudaSuccess) e = sc.get(&erow_count, 16 * RV * RV);
    if (e == cudaSuccess) e = sc.get(&erow_off, 16 * RV * RV);
    if (e == cudaSuccess) e = sc.get(&totals, 8 * 8);
    if (e != cudaSuccess) return cuda_fail(error, error_capacity, e, "flexicubes scratch");
    S3DSP_CUDA(cudaMemsetAsync(cube_row, 0x7F, 4 * kCubes, st), "memset");
    S3DSP_CUDA(cudaMemsetAsync(err_row, 0x7F, 16, st), "memset");
    launch_pdl(fc_scatter_kernel, dim3(grid_for(n, 256)), dim3(256), 0, st, coords, n, cube_row, err_row);
    launch_pdl(fc_dup_kernel, dim3(grid_for(n, 256)), dim3(256), 0, st, coords, n, cube_row, err_row);
    launch_pdl(fc_vertex_kernel, dim3((RV * RV * kVChunks + 7) / 8), dim3(256), 0, st, d_raw, cube_row, sdf, vslot,
               vattr);
    launch_pdl(fc_surface_count_kernel, dim3(R * R / 8), dim3(256), 0, st, sdf, occ, srow_count);
    launch_pdl(fc_edge_count_kernel, dim3((RV * RV + 7) / 8), dim3(256), 0, st, sdf, erow_count);
    S3DSP_LAUNCH_CHECK("flexicubes count kernels");
    size_t tb1 = 0, tb2 = 0;
    void *t1 = nullptr, *t2 = nullptr;
    e = cub::DeviceScan::ExclusiveSum(nullptr, tb1, srow_count, srow_off, R * R, st);
    if (e == cudaSuccess) e = sc.get(&t1, tb1);
    if (e == cudaSuccess) e = cub::DeviceScan::ExclusiveSum(t1, tb1, srow_count, srow_off, R * R, st);
    if (e == cudaSuccess)
        e = cub::DeviceScan::ExclusiveScan(nullptr, tb2, erow_count, erow_off, Int4Add(), make_int4(0, 0, 0, 0), RV * RV, st);
    if (e == cudaSuccess) e = sc.get(&t2, tb2);
    if (e == cudaSuccess)
        e = cub::DeviceScan::ExclusiveScan(t2, tb2, erow_count, erow_off, Int4Add(), make_int4(0, 0, 0, 0), RV * RV, st);
    if (e != cudaSuccess) return cuda_fail(error, error_capacity, e, "flexicubes row scans");
    launch_pdl(fc_totals_kernel, dim3(1), dim3(32), 0, st, srow_count, srow_off, erow_count, erow_off, err_row, totals);
    S3DSP_LAUNCH_CHECK("fc_totals_kernel");
    int64_t h_tot[8];
    S3DSP_CUDA(cudaMemcpyAsync(h_tot, totals, 7 * 8, cudaMemcpyDeviceToHost, st), "D2H");
    S3DSP_CUDA(cudaStreamSynchronize(st), "synchronize");
    {
        int kind = -1;
        int64_t first = INT64_MAX;
        for (int k = 0; k < 3; ++k)
            if (h_tot[4 + k] != kNoRow && h_tot[4 + k] < first) first = h_tot[4 + k], kind = k;
        static const char* const kMsg[3] = {"mesh extraction currently requires batch one",
                                            "mesh cube coordinate outside resolution 256",
                                            "duplicate mesh cube coordinate"};
        if (kind >= 0) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "%s", kMsg[kind]);
    }
    const int64_t ns = h_tot[0], ne = h_tot[1], nq = h_tot[2] + h_tot[3];
    auto* m = new (std::nothrow) s3dsp_mesh;
    if (!m) return fail(error, error_capacity, S3D_OUT_OF_MEMORY, "host allocation");
    m->n_surface = ns;
    m->n_edges = ne;
    m->n_faces = 2 * nq;
    const auto alloc = [&](auto** p, size_t bytes) {
        void* q = nullptr;
        const cudaError_t r = s3dsp::malloc_async(&q, bytes > 0 ? bytes : 16, st);
        *p = static_cast<std::remove_reference_t<decltype(**p)>*>(q);
        return r;
    };
    const size_t vcap = 4 * (size_t)ns;  // at most four dual vertices per surface cube
    e = alloc(&m->vertices, 12 * vcap);
    if (e == cudaSuccess) e = alloc(&m->attrs, 24 * vcap);
    if (e == cudaSuccess) e = alloc(&m->faces, 12 * (size_t)m->n_faces);
    if (e == cudaSuccess) e = alloc(&m->surface, 4 * (size_t)ns);
    if (e == cudaSuccess) e = alloc(&m->cases, 4 * (size_t)ns);
    if (e == cudaSuccess) e = alloc(&m->edges, 8 * (size_t)ne);
    int4 *onehot = nullptr, *rank = nullptr;
    float* dual_gamma = nullptr;
    int32_t *dmap = nullptr, *quads = nullptr;
    if (e == cudaSuccess) e = sc.get(&onehot, 16 * (size_t)ns);
    if (e == cudaSuccess) e = sc.get(&rank, 16 * (size_t)ns);
    if (e == cudaSuccess) e = sc.get(&dual_gamma, 4 * vcap);
    if (e == cudaSuccess) e = sc.get(&dmap, 48 * (size_t)ns);
    if (e == cudaSuccess) e = sc.get(&quads, 4 * (size_t)nq);
    if (e == cudaSuccess && ns > 0) {
        launch_pdl(fc_surface_write_kernel, dim3(R * R / 8), dim3(256), 0, st, occ, srow_off, m->surface, sidx);
        launch_pdl(fc_case_kernel, dim3(grid_for(ns, 256)), dim3(256), 0, st, m->surface, ns, occ, tables->num_dual,
                   tables->check, m->cases, onehot);
        e = cudaGetLastError();
        size_t tb3 = 0;
        void* t3 = nullptr;
        if (e == cudaSuccess)
            e = cub::DeviceScan::ExclusiveScan(nullptr, tb3, onehot, rank, Int4Add(), make_int4(0, 0, 0, 0), (int)ns, st);
        if (e == cudaSuccess) e = sc.get(&t3, tb3);
        if (e == cudaSuccess)
            e = cub::DeviceScan::ExclusiveScan(t3, tb3, onehot, rank, Int4Add(), make_int4(0, 0, 0, 0), (int)ns, st);
        if (e == cudaSuccess) {
            launch_pdl(fc_dual_kernel, dim3(grid_for(ns, 128)), dim3(128), 0, st, m->surface, ns, m->cases, onehot,
                       rank, cube_row, d_raw, sdf, vslot, vattr, tables->dmc, tables->num_dual, m->vertices, m->attrs,
                       dual_gamma, dmap, totals + 7);
            e = cudaGetLastError();
        }
    } else if (e == cudaSuccess) {
        e = cudaMemsetAsync(totals + 7, 0, 8, st);
    }
    if (e == cudaSuccess && ne > 0) {
        launch_pdl(fc_edge_write_kernel, dim3((RV * RV + 7) / 8), dim3(256), 0, st, sdf, erow_off, totals, m->edges,
                   quads);
        if (nq > 0)
            launch_pdl(fc_quad_kernel, dim3(grid_for(nq, 128)), dim3(128), 0, st, quads, nq, sidx, dmap, dual_gamma,
                       m->faces);
        e = cudaGetLastError();
    }
    int64_t nv = 0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&nv, totals + 7, 8, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        mesh_release(m, st);
        return cuda_fail(error, error_capacity, e, "flexicubes extraction");
    }
    m->n_vertices = nv;
    *out = m;
    return S3D_OK;
}

extern "C" S3DSP_API s3d_status s3dsp_mesh_info(const s3dsp_mesh* mesh, int64_t* n_vertices, int64_t* n_faces,
                                                int64_t* n_surface, int64_t* n_edges) {
    if (!mesh) return S3D_INVALID_ARGUMENT;
    if (n_vertices) *n_vertices = mesh->n_vertices;
    if (n_faces) *n_faces = mesh->n_faces;
    if (n_surface) *n_surface = mesh->n_surface;
    if (n_edges) *n_edges = mesh->n_edges;
    return S3D_OK;
}

extern "C" S3DSP_API s3d_status s3dsp_mesh_device(const s3dsp_mesh* mesh, const float** vertices,
                                                  const float** attributes, const int32_t** faces,
                                                  const int32_t** surface, const int32_t** cases,
                                                  const int32_t** edges) {
    if (!mesh) return S3D_INVALID_ARGUMENT;
    if (vertices) *vertices = mesh->vertices;
    if (attributes) *attributes = mesh->attrs;
    if (faces) *faces = mesh->faces;
    if (surface) *surface = mesh->surface;
    if (cases) *cases = mesh->cases;
    if (edges) *edges = mesh->edges;
    return S3D_OK;
}

extern "C" S3DSP_API s3d_status s3dsp_mesh_copy(s3dsp_context* ctx, const s3dsp_mesh* mesh, float* h_vertices,
                                                float* h_attributes, int32_t* h_faces, int32_t* h_surface,
                                                int32_t* h_cases, int32_t* h_edges, char* error,
                                                uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !mesh) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    cudaStream_t st = ctx->stream;
    const struct {
        void* dst;
        const void* src;
        size_t bytes;
    } copies[6] = {{h_vertices, mesh->vertices, 12 * (size_t)mesh->n_vertices},
                   {h_attributes, mesh->attrs, 24 * (size_t)mesh->n_vertices},
                   {h_faces, mesh->faces, 12 * (size_t)mesh->n_faces},
                   {h_surface, mesh->surface, 4 * (size_t)mesh->n_surface},
                   {h_cases, mesh->cases, 4 * (size_t)mesh->n_surface},
                   {h_edges, mesh->edges, 8 * (size_t)mesh->n_edges}};
    for (const auto& c : copies)
        if (c.dst && c.bytes) S3DSP_CUDA(cudaMemcpyAsync(c.dst, c.src, c.bytes, cudaMemcpyDeviceToHost, st), "D2H");
    S3DSP_CUDA(cudaStreamSynchronize(st), "synchronize");
    return S3D_OK;
}

extern "C" S3DSP_API void s3dsp_mesh_free(s3dsp_context* ctx, s3dsp_mesh* mesh) {
    if (!mesh) return;
    if (ctx) cudaSetDevice(ctx->device);
    mesh_release(mesh, ctx ? ctx->stream : nullptr);
}
