// TEST INFRASTRUCTURE ONLY — the CPU oracle for the sparse-convolution path.
//
// Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
// this library, and only as the checker (or as the timed CPU comparator). The
// product library never links, loads or falls back to it.
//
// What it restates (reference file:line in the sam3d.cpp tree):
//   * integer tables
//       - SlatTables::build            src/objects_runtime/sparse_ops.cpp:49-173
//       - MeshSubdivideTables::build   src/objects_runtime/sparse_ops.cpp:272-404
//       - GsTables::build (Swin window buckets + APE)
//                                      src/objects_runtime/sparse_ops.cpp:182-270
//     PINNED: tests compare these bit-exactly with the reference's own
//     sparse_ops.cpp compiled into oracle/_ref, and with committed goldens.
//   * float ops, in GGML graph order (GGML itself is an un-vendored submodule,
//     ggml-org/ggml @ e91ded11 / v0.23.0, absent here)
//       - SLat SubMConv3d as ONE K=27*Cin dot + bias
//                                      src/objects_runtime/slat_flow_graph.cpp:112-155
//       - mesh SubMConv3d as 27 per-offset GEMMs summed o=0..26, then bias
//                                      src/objects_runtime/mesh_decoder_graph.cpp:81-103
//       - sparse GroupNorm (all tokens of the object, eps 1e-5, then gamma/beta)
//                                      src/objects_runtime/mesh_decoder_graph.cpp:16-30
//       - LayerNorm (ggml_norm, eps 1e-6, optional affine)
//                                      src/objects_runtime/graph_builder.cpp:56-62
//       - SiLU, modulate h*(1+s)+sh    src/objects_runtime/slat_flow_graph.cpp:55-59
//       - 2x mean-pool / nearest up    src/objects_runtime/slat_flow_graph.cpp:159-190
//       - Linear (mul_mat + bias)      src/objects_runtime/graph_builder.cpp:44-54
//     PARITY UNPINNED against GGML (its CPU kernels cannot be built here); the
//     conv/norm semantics are instead cross-checked in tests against an
//     independent dense torch.conv3d / group_norm / layer_norm in float64.
//   * the coordinate pipeline before the path (src/objects_runtime/session.cpp)
//       - SS occupancy argwhere        session.cpp:1436-1441
//       - prune_surface_coords         session.cpp:122-166
//       - downsample_coords            session.cpp:168-236
//     PARITY UNPINNED against the reference: session.cpp needs GGML and cannot
//     be built here; the argwhere + prune restatement reproduces the occupancy
//     counts recorded for the reference's shipped SS fixture (69,537 -> 67,783).
//
// Layouts follow GGML's ne order with channels fastest: a feature matrix of
// (C, N) in GGML is stored here as N rows of C floats.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <numeric>
#include <random>
#include <thread>
#include <unordered_map>
#include <unordered_set>
#include <vector>

namespace {

// ---------------------------------------------------------------------------
// tiny parallel-for over [0, n) in contiguous chunks
// ---------------------------------------------------------------------------
template <class F>
void parallel_for(int64_t n, int threads, F&& body) {
    if (threads <= 0) threads = (int)std::max(1u, std::thread::hardware_concurrency());
    if (n <= 0) return;
    if (threads == 1 || n < 2 * threads) {
        body(0, n);
        return;
    }
    std::vector<std::thread> pool;
    const int64_t chunk = (n + threads - 1) / threads;
    for (int t = 0; t < threads; ++t) {
        const int64_t lo = t * chunk, hi = std::min(n, lo + chunk);
        if (lo >= hi) break;
        pool.emplace_back([&, lo, hi] { body(lo, hi); });
    }
    for (auto& th : pool) th.join();
}

struct Coord {
    int32_t b, x, y, z;
};

inline bool coord_less(const Coord& a, const Coord& c) {
    if (a.b != c.b) return a.b < c.b;
    if (a.x != c.x) return a.x < c.x;
    if (a.y != c.y) return a.y < c.y;
    return a.z < c.z;
}
inline bool coord_eq(const Coord& a, const Coord& c) {
    return a.b == c.b && a.x == c.x && a.y == c.y && a.z == c.z;
}

// Sorted unique key set with "first row" payload: a sorted vector searched by
// binary search. (The reference uses std::map; only the lookup semantics —
// exact key match, first inserted row wins — matter.)
struct SortedIndex {
    std::vector<Coord> keys;
    std::vector<int32_t> rows;

    void build(const std::vector<Coord>& pts) {
        std::vector<int32_t> order(pts.size());
        std::iota(order.begin(), order.end(), 0);
        // stable: among equal keys the smallest row comes first
        std::stable_sort(order.begin(), order.end(), [&](int32_t a, int32_t c) {
            return coord_less(pts[(size_t)a], pts[(size_t)c]);
        });
        keys.clear();
        rows.clear();
        for (int32_t i : order) {
            if (!keys.empty() && coord_eq(keys.back(), pts[(size_t)i])) continue;
            keys.push_back(pts[(size_t)i]);
            rows.push_back(i);
        }
    }
    int32_t find(const Coord& k) const {
        auto it = std::lower_bound(keys.begin(), keys.end(), k, coord_less);
        if (it == keys.end() || !coord_eq(*it, k)) return -1;
        return rows[(size_t)(it - keys.begin())];
    }
};

// Offset o in [0,27): (dx, dy, dz) = (o/9-1, (o/3)%3-1, o%3-1) on (x, y, z).
// sparse_ops.cpp:132 (SLat) and :351-352 / :375-377 (mesh).
inline void offset_delta(int o, int& dx, int& dy, int& dz) {
    dx = o / 9 - 1;
    dy = (o / 3) % 3 - 1;
    dz = o % 3 - 1;
}

inline int64_t floor_div2(int64_t v) { return v >= 0 ? v / 2 : -((-v + 1) / 2); }

}  // namespace

extern "C" {

// ---------------------------------------------------------------------------
// SlatTables restatement (sparse_ops.cpp:49-173, without the APE table)
//
// coords: nf rows of (b, x, y, z). Outputs sized by the caller for nc <= nf:
//   fine_to_coarse[nf], coarse_children[8*nc], coarse_inv_count[nc],
//   conv_fine[27*nf] (sentinel nf), conv_coarse[27*nc] (sentinel nc),
//   coarse_coords[4*nc] (row order; not part of the reference struct but
//   useful for tests). Returns nc, or -1 when nf <= 0 (sparse_ops.cpp:51).
// ---------------------------------------------------------------------------
int64_t oracle_slat_tables(const int32_t* coords, int64_t nf, int32_t* fine_to_coarse,
                           int32_t* coarse_children, float* coarse_inv_count,
                           int32_t* conv_fine, int32_t* conv_coarse, int32_t* coarse_coords) {
    if (nf <= 0) return -1;
    std::vector<Coord> fine((size_t)nf), coarse_of((size_t)nf);
    for (int64_t i = 0; i < nf; ++i) {
        const int32_t* c = coords + 4 * i;
        fine[(size_t)i] = {c[0], c[1], c[2], c[3]};
        // C++ integer division truncates toward zero (sparse_ops.cpp:63-64)
        coarse_of[(size_t)i] = {c[0], c[1] / 2, c[2] / 2, c[3] / 2};
    }
    // coarse rows = sorted unique coarse keys (sparse_ops.cpp:53-71)
    SortedIndex coarse;
    coarse.build(coarse_of);
    const int64_t nc = (int64_t)coarse.keys.size();
    for (int64_t c = 0; c < nc; ++c) coarse.rows[(size_t)c] = (int32_t)c;  // row id = rank
    std::vector<int32_t> counts((size_t)nc, 0);
    for (int64_t i = 0; i < nf; ++i) {
        const int32_t c = coarse.find(coarse_of[(size_t)i]);
        fine_to_coarse[i] = c;
        // children in increasing fine row order, at most 8 kept (:84-90)
        const int32_t slot = counts[(size_t)c]++;
        if (slot < 8) coarse_children[(size_t)c * 8 + slot] = (int32_t)i;
    }
    for (int64_t c = 0; c < nc; ++c) {
        for (int32_t j = std::min(counts[(size_t)c], 8); j < 8; ++j)
            coarse_children[(size_t)c * 8 + j] = (int32_t)nf;  // sentinel = zero row
        // torch scatter_reduce "mean" counts the initial zero too (:93-96)
        coarse_inv_count[c] = 1.0f / (float)(counts[(size_t)c] + 1);
        if (coarse_coords) {
            const Coord& k = coarse.keys[(size_t)c];
            coarse_coords[4 * c + 0] = k.b;
            coarse_coords[4 * c + 1] = k.x;
            coarse_coords[4 * c + 2] = k.y;
            coarse_coords[4 * c + 3] = k.z;
        }
    }
    // submanifold neighbour tables (sparse_ops.cpp:117-142): only the first
    // row of a duplicated key is filled; every other entry is the sentinel.
    SortedIndex fidx;
    fidx.build(fine);
    auto fill = [](const SortedIndex& idx, int64_t n, int32_t* table) {
        for (int64_t i = 0; i < 27 * n; ++i) table[i] = (int32_t)n;
        for (size_t u = 0; u < idx.keys.size(); ++u) {
            const Coord& k = idx.keys[u];
            const int32_t row = idx.rows[u];
            for (int o = 0; o < 27; ++o) {
                int dx, dy, dz;
                offset_delta(o, dx, dy, dz);
                const int32_t hit = idx.find({k.b, k.x + dx, k.y + dy, k.z + dz});
                if (hit >= 0) table[(size_t)row * 27 + o] = hit;
            }
        }
    };
    fill(fidx, nf, conv_fine);
    fill(coarse, nc, conv_coarse);
    return nc;
}

// ---------------------------------------------------------------------------
// MeshSubdivideTables restatement (sparse_ops.cpp:272-404)
//
// Child row = parent*8 + (xb*4 + yb*2 + zb), coords 2p + bits (:334-343).
// Neighbours are derived here from the CHILD geometry (floor division of the
// neighbour child coordinate by two gives its parent), an independent route
// to the same table the reference builds from 27 parent probes plus its
// adjacent_offset/adjacent_child tables (:346-402). Missing -> -1.
// Returns 1, or 0 on count <= 0, count > INT32_MAX/8, or a duplicate parent.
// ---------------------------------------------------------------------------
int32_t oracle_mesh_subdivide(const int32_t* parents, int64_t count, int32_t* child_coords,
                              int32_t* neighbors) {
    if (!parents || count <= 0 || count > INT32_MAX / 8) return 0;
    std::vector<Coord> pts((size_t)count);
    for (int64_t p = 0; p < count; ++p)
        pts[(size_t)p] = {parents[4 * p], parents[4 * p + 1], parents[4 * p + 2], parents[4 * p + 3]};
    SortedIndex idx;
    idx.build(pts);
    if ((int64_t)idx.keys.size() != count) return 0;  // duplicate parent (:325-333)
    for (int64_t p = 0; p < count; ++p) {
        const Coord& P = pts[(size_t)p];
        for (int j = 0; j < 8; ++j) {
            int32_t* cc = child_coords + 4 * (p * 8 + j);
            cc[0] = P.b;
            cc[1] = P.x * 2 + j / 4;
            cc[2] = P.y * 2 + (j / 2) % 2;
            cc[3] = P.z * 2 + j % 2;
        }
    }
    for (int64_t p = 0; p < count; ++p) {
        const Coord& P = pts[(size_t)p];
        for (int j = 0; j < 8; ++j) {
            const int64_t cx = (int64_t)P.x * 2 + j / 4, cy = (int64_t)P.y * 2 + (j / 2) % 2,
                          cz = (int64_t)P.z * 2 + j % 2;
            int32_t* row = neighbors + (p * 8 + j) * 27;
            for (int o = 0; o < 27; ++o) {
                int dx, dy, dz;
                offset_delta(o, dx, dy, dz);
                const int64_t tx = cx + dx, ty = cy + dy, tz = cz + dz;
                const int32_t hit = idx.find({P.b, (int32_t)floor_div2(tx), (int32_t)floor_div2(ty),
                                              (int32_t)floor_div2(tz)});
                if (hit < 0) {
                    row[o] = -1;
                } else {
                    const int bits = (int)((tx - 2 * floor_div2(tx)) * 4 + (ty - 2 * floor_div2(ty)) * 2 +
                                           (tz - 2 * floor_div2(tz)));
                    row[o] = hit * 8 + bits;
                }
            }
        }
    }
    return 1;
}

// ---------------------------------------------------------------------------
// Register-blocked f32 micro-kernel shared by both conv formulations:
// acc[i][j] (+)= sum_k a_i[k] * wt[k][j] for 4 rows i and a 32-wide slab of
// output channels j, k ascending (one sequential f32 sum per element).
// wt is K-major [K][cout]. Rows with a null pointer contribute zeros.
// ---------------------------------------------------------------------------
constexpr int kRowBlk = 4;
constexpr int kColBlk = 32;

static inline void micro_axpy(const float* const a[kRowBlk], const float* wt, int64_t K,
                              int64_t cout, int64_t co0, int64_t ncol,
                              float acc[kRowBlk][kColBlk]) {
    for (int i = 0; i < kRowBlk; ++i)
        for (int j = 0; j < kColBlk; ++j) acc[i][j] = 0.0f;
    if (ncol == kColBlk) {
        for (int64_t k = 0; k < K; ++k) {
            const float* wk = wt + k * cout + co0;
            for (int i = 0; i < kRowBlk; ++i) {
                const float av = a[i] ? a[i][k] : 0.0f;
                for (int j = 0; j < kColBlk; ++j) acc[i][j] += av * wk[j];
            }
        }
    } else {
        for (int64_t k = 0; k < K; ++k) {
            const float* wk = wt + k * cout + co0;
            for (int i = 0; i < kRowBlk; ++i) {
                const float av = a[i] ? a[i][k] : 0.0f;
                for (int j = 0; j < ncol; ++j) acc[i][j] += av * wk[j];
            }
        }
    }
}

static void transpose_w(const float* w, int64_t rows, int64_t cols, std::vector<float>& wt) {
    wt.resize((size_t)(rows * cols));
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t c = 0; c < cols; ++c) wt[(size_t)(c * rows + r)] = w[r * cols + c];
}

// ---------------------------------------------------------------------------
// SLat SubMConv3d, GGML order (slat_flow_graph.cpp:112-155)
//   xc = concat(feat, zero row); g = get_rows(xc, idx[27n]) -> (27*Cin, n);
//   out = mul_mat(W[Cout, 27*Cin], g) + bias.
// Each output element is ONE K = 27*Cin dot product in (offset, channel)
// order, then the bias add. nbr entries outside [0, n_in) read the zero row
// (the reference's sentinel is exactly n_in). accum64 != 0 accumulates in
// double (a high-precision check); otherwise one sequential f32 sum.
// ---------------------------------------------------------------------------
void oracle_subm_conv_slat(const float* feat, int64_t n_in, int64_t cin, const int32_t* nbr,
                           int64_t n_out, const float* w, const float* bias, int64_t cout,
                           float* out, int32_t accum64, int32_t threads) {
    const int64_t K = 27 * cin;
    if (accum64) {
        parallel_for(n_out, threads, [&](int64_t lo, int64_t hi) {
            for (int64_t r = lo; r < hi; ++r)
                for (int64_t co = 0; co < cout; ++co) {
                    double acc = 0.0;
                    for (int o = 0; o < 27; ++o) {
                        const int32_t s = nbr[r * 27 + o];
                        if (s < 0 || s >= n_in) continue;
                        const float* xr = feat + (int64_t)s * cin;
                        const float* wr = w + co * K + o * cin;
                        for (int64_t k = 0; k < cin; ++k) acc += (double)wr[k] * (double)xr[k];
                    }
                    out[r * cout + co] = (float)acc + (bias ? bias[co] : 0.0f);
                }
        });
        return;
    }
    std::vector<float> wt;
    transpose_w(w, cout, K, wt);  // [K][cout]
    const int64_t nblk = (n_out + kRowBlk - 1) / kRowBlk;
    parallel_for(nblk, threads, [&](int64_t lo, int64_t hi) {
        std::vector<float> g((size_t)(kRowBlk * K));
        float acc[kRowBlk][kColBlk];
        for (int64_t b = lo; b < hi; ++b) {
            const float* a[kRowBlk];
            for (int i = 0; i < kRowBlk; ++i) {
                const int64_t r = b * kRowBlk + i;
                a[i] = nullptr;
                if (r >= n_out) continue;
                float* gi = g.data() + (size_t)i * K;
                for (int o = 0; o < 27; ++o) {
                    const int32_t s = nbr[r * 27 + o];
                    if (s >= 0 && s < n_in)
                        std::memcpy(gi + o * cin, feat + (int64_t)s * cin, (size_t)cin * 4);
                    else
                        std::memset(gi + o * cin, 0, (size_t)cin * 4);
                }
                a[i] = gi;
            }
            for (int64_t co0 = 0; co0 < cout; co0 += kColBlk) {
                const int64_t nc = std::min<int64_t>(kColBlk, cout - co0);
                micro_axpy(a, wt.data(), K, cout, co0, nc, acc);
                for (int i = 0; i < kRowBlk; ++i) {
                    const int64_t r = b * kRowBlk + i;
                    if (r >= n_out) continue;
                    for (int64_t j = 0; j < nc; ++j)
                        out[r * cout + co0 + j] = acc[i][j] + (bias ? bias[co0 + j] : 0.0f);
                }
            }
        }
    });
}

// ---------------------------------------------------------------------------
// mesh SubMConv3d, GGML order (mesh_decoder_graph.cpp:81-103)
//   for o in 0..kvol-1: v_o = mul_mat(W_o[Cout,Cin], get_rows(x, idx_o) * mask_o)
//   sum = ((v_0 + v_1) + v_2) + ...; out = sum + bias
// idx/mask come from neighbors[row*27+o] (mesh_decoder_graph.cpp:68-79):
// idx = src<0 ? 0 : src, mask = src<0 ? 0 : 1. The gathered row index is
// (src >> gather_shift): gather_shift = 3 reads the PARENT row of a child,
// which equals reading the child of repeat_children(x) (:32-38). kvol == 1
// is the 1x1 skip conv: no gather, row r reads x[r >> gather_shift].
// w_packed is [kvol][Cout][Cin] (convert_sam3d_to_gguf.py:481-492 layout).
// ---------------------------------------------------------------------------
void oracle_subm_conv_mesh(const float* feat, int64_t n_in, int64_t cin, const int32_t* nbr,
                           int32_t kvol, int32_t gather_shift, int64_t n_out,
                           const float* w_packed, const float* bias, int64_t cout, float* out,
                           int32_t accum64, int32_t threads) {
    auto src_row = [&](int64_t r, int o) -> const float* {
        if (kvol == 1) return feat + (r >> gather_shift) * cin;
        const int32_t s = nbr[r * 27 + o];
        if (s < 0) return nullptr;  // masked to zero
        return feat + (int64_t)(s >> gather_shift) * cin;
    };
    if (accum64) {
        parallel_for(n_out, threads, [&](int64_t lo, int64_t hi) {
            std::vector<double> sum((size_t)cout);
            for (int64_t r = lo; r < hi; ++r) {
                for (int o = 0; o < kvol; ++o) {
                    const float* xr = src_row(r, o);
                    for (int64_t co = 0; co < cout; ++co) {
                        double acc = 0.0;
                        if (xr) {
                            const float* wr = w_packed + ((int64_t)o * cout + co) * cin;
                            for (int64_t k = 0; k < cin; ++k) acc += (double)wr[k] * (double)xr[k];
                        }
                        sum[(size_t)co] = o == 0 ? acc : sum[(size_t)co] + acc;
                    }
                }
                for (int64_t co = 0; co < cout; ++co)
                    out[r * cout + co] = (float)sum[(size_t)co] + (bias ? bias[co] : 0.0f);
            }
        });
        return;
    }
    std::vector<float> wt((size_t)(kvol * cin * cout));
    for (int o = 0; o < kvol; ++o) {
        std::vector<float> t;
        transpose_w(w_packed + (int64_t)o * cout * cin, cout, cin, t);
        std::memcpy(wt.data() + (size_t)o * cin * cout, t.data(), t.size() * 4);
    }
    const int64_t nblk = (n_out + kRowBlk - 1) / kRowBlk;
    parallel_for(nblk, threads, [&](int64_t lo, int64_t hi) {
        float acc[kRowBlk][kColBlk];
        std::vector<float> sum((size_t)(kRowBlk * cout));
        for (int64_t b = lo; b < hi; ++b) {
            for (int o = 0; o < kvol; ++o) {
                const float* a[kRowBlk];
                for (int i = 0; i < kRowBlk; ++i) {
                    const int64_t r = b * kRowBlk + i;
                    a[i] = r < n_out ? src_row(r, o) : nullptr;
                }
                for (int64_t co0 = 0; co0 < cout; co0 += kColBlk) {
                    const int64_t nc = std::min<int64_t>(kColBlk, cout - co0);
                    micro_axpy(a, wt.data() + (size_t)o * cin * cout, cin, cout, co0, nc, acc);
                    for (int i = 0; i < kRowBlk; ++i)
                        for (int64_t j = 0; j < nc; ++j) {
                            float& s = sum[(size_t)(i * cout + co0 + j)];
                            s = o == 0 ? acc[i][j] : s + acc[i][j];
                        }
                }
            }
            for (int i = 0; i < kRowBlk; ++i) {
                const int64_t r = b * kRowBlk + i;
                if (r >= n_out) continue;
                for (int64_t co = 0; co < cout; ++co)
                    out[r * cout + co] = sum[(size_t)(i * cout + co)] + (bias ? bias[co] : 0.0f);
            }
        }
    });
    (void)n_in;
}

// ---------------------------------------------------------------------------
// Linear (gb_linear: mul_mat + bias, graph_builder.cpp:44-54); W is [Cout][Cin].
// row_shift reads x[r >> row_shift] (the 1x1 skip on repeated parents).
// ---------------------------------------------------------------------------
void oracle_linear(const float* x, int64_t n, int64_t cin, int32_t row_shift, const float* w,
                   const float* bias, int64_t cout, float* out, int32_t threads) {
    oracle_subm_conv_mesh(x, n, cin, nullptr, 1, row_shift, n, w, bias, cout, out, 0, threads);
}

// ---------------------------------------------------------------------------
// GroupNorm over every token of one object (mesh_decoder_graph.cpp:16-30):
// groups split C into equal consecutive channel ranges; mean and variance in
// double over (tokens x channels-of-group), variance = mean((x-mean)^2),
// y = (x-mean) * (1/sqrtf(var+eps)), then * gamma[c] + beta[c].
// Optional silu fuses ggml_silu (mesh_decoder_graph.cpp:109, :121).
// ---------------------------------------------------------------------------
void oracle_group_norm(const float* x, int64_t n, int64_t c, int32_t groups, float eps,
                       const float* gamma, const float* beta, int32_t silu, float* out) {
    const int64_t gs = c / groups;
    for (int32_t g = 0; g < groups; ++g) {
        double sum = 0.0;
        for (int64_t r = 0; r < n; ++r)
            for (int64_t k = g * gs; k < (g + 1) * gs; ++k) sum += x[r * c + k];
        const double cnt = (double)n * (double)gs;
        const float mean = (float)(sum / cnt);
        double sum2 = 0.0;
        for (int64_t r = 0; r < n; ++r)
            for (int64_t k = g * gs; k < (g + 1) * gs; ++k) {
                const float v = x[r * c + k] - mean;
                sum2 += (double)v * (double)v;
            }
        const float scale = 1.0f / sqrtf((float)(sum2 / cnt) + eps);
        for (int64_t r = 0; r < n; ++r)
            for (int64_t k = g * gs; k < (g + 1) * gs; ++k) {
                float v = (x[r * c + k] - mean) * scale;
                if (gamma) v *= gamma[k];
                if (beta) v += beta[k];
                if (silu) v = v / (1.0f + expf(-v));
                out[r * c + k] = v;
            }
    }
}

// ---------------------------------------------------------------------------
// LayerNorm per token (ggml_norm + optional mul/add, graph_builder.cpp:56-62),
// optional modulate h*(1+scale)+shift (slat_flow_graph.cpp:55-59) and SiLU.
// ---------------------------------------------------------------------------
void oracle_layer_norm(const float* x, int64_t n, int64_t c, float eps, const float* gamma,
                       const float* beta, const float* mod_scale, const float* mod_shift,
                       int32_t silu, float* out) {
    for (int64_t r = 0; r < n; ++r) {
        const float* xr = x + r * c;
        double sum = 0.0;
        for (int64_t k = 0; k < c; ++k) sum += xr[k];
        const float mean = (float)(sum / (double)c);
        double sum2 = 0.0;
        for (int64_t k = 0; k < c; ++k) {
            const float v = xr[k] - mean;
            sum2 += (double)v * (double)v;
        }
        const float scale = 1.0f / sqrtf((float)(sum2 / (double)c) + eps);
        for (int64_t k = 0; k < c; ++k) {
            float v = (xr[k] - mean) * scale;
            if (gamma) v *= gamma[k];
            if (beta) v += beta[k];
            if (mod_scale) v = v * mod_scale[k] + v;
            if (mod_shift) v += mod_shift[k];
            if (silu) v = v / (1.0f + expf(-v));
            out[r * c + k] = v;
        }
    }
}

// SparseDownsample mean (slat_flow_graph.cpp:159-183): out[c] = (sum over the
// 8 children slots of xc[child]) * inv_count[c]; slots == nf read zeros.
void oracle_downsample_mean(const float* x, int64_t nf, int64_t ch, const int32_t* children,
                            const float* inv_count, int64_t nc, float* out) {
    for (int64_t c = 0; c < nc; ++c) {
        for (int64_t k = 0; k < ch; ++k) {
            float s = 0.0f;
            for (int j = 0; j < 8; ++j) {
                const int32_t f = children[c * 8 + j];
                const float v = (f >= 0 && f < nf) ? x[(int64_t)f * ch + k] : 0.0f;
                s = j == 0 ? v : s + v;
            }
            out[c * ch + k] = s * inv_count[c];
        }
    }
}

// SparseUpsample nearest (slat_flow_graph.cpp:186-190): out[i] = x[f2c[i]].
void oracle_upsample_nearest(const float* x, int64_t nc, int64_t ch, const int32_t* f2c,
                             int64_t nf, float* out) {
    for (int64_t i = 0; i < nf; ++i) {
        const int32_t c = f2c[i];
        for (int64_t k = 0; k < ch; ++k)
            out[i * ch + k] = (c >= 0 && c < nc) ? x[(int64_t)c * ch + k] : 0.0f;
    }
}

// ---------------------------------------------------------------------------
// coordinate pipeline (src/objects_runtime/session.cpp)
// ---------------------------------------------------------------------------
static inline uint64_t coord_key(int32_t b, int32_t x, int32_t y, int32_t z) {
    // the reference's coordinate_key (session.cpp:122-127)
    return ((uint64_t)(uint32_t)b << 48) | ((uint64_t)(uint32_t)x << 32) | ((uint64_t)(uint32_t)y << 16) |
           ((uint64_t)(uint32_t)z & 0xffffu);
}

// occupancy argwhere (session.cpp:1436-1441): occ[(x*ny + y)*nz + z] > 0 ->
// row (batch, x, y, z), x-major. Returns the row count.
int64_t oracle_occupancy_coords(const float* occ, int32_t nx, int32_t ny, int32_t nz, int32_t batch,
                                int32_t* out) {
    int64_t n = 0;
    for (int32_t x = 0; x < nx; ++x)
        for (int32_t y = 0; y < ny; ++y)
            for (int32_t z = 0; z < nz; ++z)
                if (occ[((int64_t)x * ny + y) * nz + z] > 0.0f) {
                    out[4 * n + 0] = batch;
                    out[4 * n + 1] = x;
                    out[4 * n + 2] = y;
                    out[4 * n + 3] = z;
                    ++n;
                }
    return n;
}

// prune_surface_coords (session.cpp:129-166): keep a row iff some cell of its
// (2d+1)^3 neighbourhood is unoccupied, input order kept. Returns the count.
int64_t oracle_prune_surface(const int32_t* coords, int64_t n, int32_t d, int32_t* out) {
    std::unordered_set<uint64_t> occ;
    occ.reserve((size_t)n * 2);
    for (int64_t i = 0; i < n; ++i) occ.insert(coord_key(coords[4 * i], coords[4 * i + 1], coords[4 * i + 2], coords[4 * i + 3]));
    int64_t m = 0;
    for (int64_t i = 0; i < n; ++i) {
        const int32_t* c = coords + 4 * i;
        bool surface = false;
        for (int dx = -d; dx <= d && !surface; ++dx)
            for (int dy = -d; dy <= d && !surface; ++dy)
                for (int dz = -d; dz <= d && !surface; ++dz)
                    surface = occ.find(coord_key(c[0], c[1] + dx, c[2] + dy, c[3] + dz)) == occ.end();
        if (surface) {
            std::memcpy(out + 4 * m, c, 16);
            ++m;
        }
    }
    return m;
}

// downsample_coords (session.cpp:168-236): above max_coords rows, rescale each
// axis by 1/factor about the box centre (double arithmetic, round half up,
// clamped), keep first occurrences, and above max_coords again keep
// max_coords rows chosen by std::shuffle with std::mt19937(seed). Returns the
// count; out holds n rows at most. Unfused multiply-add, as the reference is
// built (-ffp-contract=off, CMakeLists.txt:65).
__attribute__((optimize("fp-contract=off")))
int64_t oracle_downsample_coords(const int32_t* coords, int64_t n, int64_t max_coords, int32_t factor,
                                 uint32_t seed, int32_t* out) {
    if (n <= max_coords) {
        std::memcpy(out, coords, (size_t)n * 16);
        return n;
    }
    int32_t lo[3] = {coords[1], coords[2], coords[3]}, hi[3] = {coords[1], coords[2], coords[3]};
    for (int64_t i = 1; i < n; ++i)
        for (int c = 0; c < 3; ++c) {
            lo[c] = std::min(lo[c], coords[4 * i + c + 1]);
            hi[c] = std::max(hi[c], coords[4 * i + c + 1]);
        }
    double target[3], tmin[3];
    int32_t tmin_i[3], tmax_i[3];
    for (int c = 0; c < 3; ++c) {
        const double original = (double)(hi[c] - lo[c] + 1);
        target[c] = original / (double)factor;
        const double offset = (original - target[c]) * 0.5;
        tmin[c] = (double)lo[c] + offset;
        const double tmax = tmin[c] + target[c] - 1.0;
        tmin_i[c] = (int32_t)tmin[c];  // truncation toward zero, as torch .int()
        tmax_i[c] = (int32_t)tmax;
    }
    std::vector<int32_t> uniq;
    std::unordered_set<uint64_t> seen;
    seen.reserve((size_t)n * 2);
    for (int64_t i = 0; i < n; ++i) {
        const int32_t* p = coords + 4 * i;
        int32_t o[4] = {p[0], 0, 0, 0};
        for (int c = 0; c < 3; ++c) {
            const double denom = (double)(hi[c] - lo[c]);
            const double normalized = denom > 0.0 ? ((double)p[c + 1] - lo[c]) / denom : 0.0;
            const double value = normalized * (target[c] - 1.0) + tmin[c];
            int64_t r = (int64_t)std::floor(value + 0.5);
            r = std::max<int64_t>(r, tmin_i[c]);
            r = std::min<int64_t>(r, tmax_i[c]);
            o[c + 1] = (int32_t)r;
        }
        if (seen.insert(coord_key(o[0], o[1], o[2], o[3])).second) uniq.insert(uniq.end(), o, o + 4);
    }
    const int64_t un = (int64_t)uniq.size() / 4;
    if (un > max_coords) {
        std::mt19937 rng(seed);
        std::vector<size_t> order((size_t)un);
        std::iota(order.begin(), order.end(), 0);
        std::shuffle(order.begin(), order.end(), rng);
        for (int64_t j = 0; j < max_coords; ++j) std::memcpy(out + 4 * j, &uniq[order[(size_t)j] * 4], 16);
        return max_coords;
    }
    std::memcpy(out, uniq.data(), (size_t)un * 16);
    return un;
}

// ---------------------------------------------------------------------------
// GS decoder Swin window tables (sparse_ops.cpp:182-270)
// ---------------------------------------------------------------------------
// Windows of side `window` over coords shifted by `shift` (C division); a
// window's id is the order of its first token; tokens are grouped by window
// (window-id order, table order inside), and windows are laid out by token
// count ascending, window-id order within a count. bkt_idx[row] = original
// token, bwd_idx[token] = row; buckets[3*k] = {len, first row, windows}.
// Returns the bucket count, or -1 for n <= 0.
int64_t oracle_gs_window_tables(const int32_t* coords, int64_t n, int32_t shift, int32_t window, int32_t* bkt_idx,
                                int32_t* bwd_idx, int32_t* buckets) {
    if (n <= 0) return -1;
    struct K {
        int32_t b, x, y, z;
        bool operator==(const K& o) const { return b == o.b && x == o.x && y == o.y && z == o.z; }
    };
    struct H {
        size_t operator()(const K& k) const {
            return std::hash<uint64_t>()(((uint64_t)(uint32_t)k.b << 32) ^ ((uint64_t)(uint32_t)k.x << 21) ^
                                         ((uint64_t)(uint32_t)k.y << 10) ^ (uint64_t)(uint32_t)k.z);
        }
    };
    std::unordered_map<K, int32_t, H> ids;
    std::vector<int32_t> wid((size_t)n);
    for (int64_t i = 0; i < n; ++i) {
        const K k{coords[4 * i], (coords[4 * i + 1] + shift) / window, (coords[4 * i + 2] + shift) / window,
                  (coords[4 * i + 3] + shift) / window};
        wid[(size_t)i] = ids.emplace(k, (int32_t)ids.size()).first->second;
    }
    const int32_t nw = (int32_t)ids.size();
    // tokens per window and each window's tokens in table order (counting sort)
    std::vector<int32_t> cnt((size_t)nw, 0), start((size_t)nw + 1, 0), tokens((size_t)n);
    for (int64_t i = 0; i < n; ++i) ++cnt[(size_t)wid[(size_t)i]];
    for (int32_t w = 0; w < nw; ++w) start[(size_t)w + 1] = start[(size_t)w] + cnt[(size_t)w];
    std::vector<int32_t> fill(start.begin(), start.end() - 1);
    for (int64_t i = 0; i < n; ++i) tokens[(size_t)fill[(size_t)wid[(size_t)i]]++] = (int32_t)i;
    // windows by (token count, id)
    std::vector<int32_t> wins((size_t)nw);
    std::iota(wins.begin(), wins.end(), 0);
    std::stable_sort(wins.begin(), wins.end(), [&](int32_t a, int32_t b) { return cnt[(size_t)a] < cnt[(size_t)b]; });
    int32_t row = 0;
    int64_t nb = 0;
    for (size_t k = 0; k < wins.size(); ++k) {
        const int32_t w = wins[k];
        const int32_t len = cnt[(size_t)w];
        if (k == 0 || len != cnt[(size_t)wins[k - 1]]) {
            buckets[3 * nb + 0] = len;
            buckets[3 * nb + 1] = row;
            buckets[3 * nb + 2] = 0;
            ++nb;
        }
        ++buckets[3 * (nb - 1) + 2];
        for (int32_t j = 0; j < len; ++j) {
            const int32_t t = tokens[(size_t)(start[(size_t)w] + j)];
            bkt_idx[row] = t;
            bwd_idx[t] = row;
            ++row;
        }
    }
    return nb;
}

// AbsolutePositionEmbedder (sparse_ops.cpp:242-262): per token and axis,
// channels/6 sines then channels/6 cosines of coordinate * 10000^(-i/(channels/6)).
void oracle_ape(const int32_t* coords, int64_t n, int32_t channels, float* out) {
    const int f = channels / 6;
    std::vector<float> freq((size_t)f);
    for (int i = 0; i < f; ++i) freq[(size_t)i] = 1.0f / powf(10000.0f, (float)i / (float)f);
    for (int64_t t = 0; t < n; ++t)
        for (int a = 0; a < 3; ++a) {
            const float v = (float)coords[4 * t + 1 + a];
            float* o = out + (size_t)t * channels + (size_t)a * 2 * f;
            for (int i = 0; i < f; ++i) {
                o[i] = sinf(v * freq[(size_t)i]);
                o[f + i] = cosf(v * freq[(size_t)i]);
            }
        }
}

// ---------------------------------------------------------------------------
// FlexiCubes extraction at 256^3: SparseFeatures2Mesh + inference FlexiCubes
// (src/objects_runtime/mesh_extractor.cpp:95-377), restated over dense grids
// (cube -> row, vertex -> SDF, vertex -> attribute slot) in the arithmetic
// order of the reference: a vertex's sums run over its cubes in ascending row
// order; the dual-vertex, quad and face orders are the reference's. The DMC
// tables (dmc [256][4][7], num_dual [256], check [256][5]) are inputs.
// Results stay in a process-wide buffer until the next call
// (oracle_flexicubes_fetch copies them out).
// ---------------------------------------------------------------------------
namespace fcx {
constexpr int R = 256, RV = 257, RAW = 101;
// corner c = (c & 1, c >> 1 & 1, c >> 2 & 1); edge e joins kEdge[e][0] -> kEdge[e][1]
constexpr int kCorner[8][3] = {{0, 0, 0}, {1, 0, 0}, {0, 1, 0}, {1, 1, 0}, {0, 0, 1}, {1, 0, 1}, {0, 1, 1}, {1, 1, 1}};
constexpr int kEdge[12][2] = {{0, 1}, {1, 5}, {4, 5}, {0, 4}, {2, 3}, {3, 7}, {6, 7}, {2, 6}, {2, 0}, {3, 1}, {7, 5}, {6, 4}};
inline int64_t vid(int x, int y, int z) { return ((int64_t)x * RV + y) * RV + z; }
inline int64_t cid(int x, int y, int z) { return ((int64_t)x * R + y) * R + z; }
struct Mesh {
    std::vector<float> vertices, attrs;
    std::vector<int32_t> faces, surface, cases, edges;
};
Mesh g_mesh;
}  // namespace fcx

// Returns 0, or -1 bad arguments, -2 batch != 0, -3 coordinate outside
// [0, 256), -4 duplicate coordinate (the reference's three input errors).
// counts: {dual vertices, triangles, surface cubes, surface edges}.
__attribute__((optimize("fp-contract=off")))
int32_t oracle_flexicubes(const float* raw, const int32_t* coords, int64_t n, const int8_t* dmc,
                          const int8_t* num_dual, const int16_t* check, int64_t* counts) {
    using namespace fcx;
    g_mesh = Mesh{};
    if (!raw || !coords || n <= 0 || n > INT32_MAX || !dmc || !num_dual || !check) return -1;
    std::vector<int32_t> cube_row((size_t)R * R * R, -1);
    for (int64_t r = 0; r < n; ++r) {
        const int32_t* c = coords + 4 * r;
        if (c[0] != 0) return -2;
        if (c[1] < 0 || c[2] < 0 || c[3] < 0 || c[1] >= R || c[2] >= R || c[3] >= R) return -3;
        int32_t& slot = cube_row[(size_t)cid(c[1], c[2], c[3])];
        if (slot >= 0) return -4;
        slot = (int32_t)r;
    }
    // per-vertex means, computed once by the lowest-row cube holding the vertex
    const size_t nv = (size_t)RV * RV * RV;
    std::vector<float> sdf(nv, 1.0f);
    std::vector<int32_t> vslot(nv, -1);
    std::vector<float> vattr((size_t)n * 8 * 9);
    for (int64_t r = 0; r < n; ++r)
        for (int corner = 0; corner < 8; ++corner) {
            const int x = coords[4 * r + 1] + kCorner[corner][0], y = coords[4 * r + 2] + kCorner[corner][1],
                      z = coords[4 * r + 3] + kCorner[corner][2];
            int32_t rows[8], ks[8], m = 0;
            for (int k = 0; k < 8; ++k) {
                const int cx = x - kCorner[k][0], cy = y - kCorner[k][1], cz = z - kCorner[k][2];
                if (cx < 0 || cy < 0 || cz < 0 || cx >= R || cy >= R || cz >= R) continue;
                const int32_t row = cube_row[(size_t)cid(cx, cy, cz)];
                if (row < 0) continue;
                int j = m++;
                for (; j > 0 && rows[j - 1] > row; --j) rows[j] = rows[j - 1], ks[j] = ks[j - 1];
                rows[j] = row, ks[j] = k;
            }
            if (rows[0] != r) continue;  // owned by a lower row
            float sum[10] = {};
            for (int j = 0; j < m; ++j) {
                const float* f = raw + (size_t)rows[j] * RAW;
                const int k = ks[j];
                sum[0] += f[k] - 1.0f / R;
                for (int a = 0; a < 3; ++a) sum[1 + a] += f[8 + 3 * k + a];
                for (int ch = 0; ch < 6; ++ch) sum[4 + ch] += f[53 + 6 * k + ch];
            }
            float mean[10];
            for (int ch = 0; ch < 10; ++ch) mean[ch] = sum[ch] / (float)m;
            const int64_t v = vid(x, y, z);
            sdf[(size_t)v] = mean[0];
            const int64_t slot = r * 8 + corner;
            float* o = vattr.data() + slot * 9;
            const int p[3] = {x, y, z};
            for (int a = 0; a < 3; ++a)
                o[a] = (float)p[a] / R - 0.5f + (1.0f / (R * 2.0f)) * std::tanh(mean[1 + a]);
            for (int ch = 0; ch < 6; ++ch) o[3 + ch] = 1.0f / (1.0f + std::exp(-mean[4 + ch]));
            vslot[(size_t)v] = (int32_t)slot;
        }
    const auto vertex_attr = [&](int64_t v, float out[9]) {
        const int32_t s = vslot[(size_t)v];
        if (s >= 0) {
            std::memcpy(out, vattr.data() + (size_t)s * 9, 9 * sizeof(float));
            return;
        }
        const int p[3] = {(int)(v / ((int64_t)RV * RV)), (int)(v / RV % RV), (int)(v % RV)};
        for (int a = 0; a < 3; ++a) out[a] = (float)p[a] / R - 0.5f;
        for (int ch = 0; ch < 6; ++ch) out[3 + ch] = 0.5f;
    };
    // surface cubes in dense (x, y, z) order
    std::vector<uint8_t> occ((size_t)R * R * R);
    std::vector<int32_t> sidx((size_t)R * R * R, -1);
    std::vector<int32_t>& surf = g_mesh.surface;
    for (int x = 0; x < R; ++x)
        for (int y = 0; y < R; ++y)
            for (int z = 0; z < R; ++z) {
                unsigned bits = 0;
                for (int k = 0; k < 8; ++k)
                    if (sdf[(size_t)vid(x + kCorner[k][0], y + kCorner[k][1], z + kCorner[k][2])] < 0.0f) bits |= 1u << k;
                const int64_t c = cid(x, y, z);
                occ[(size_t)c] = (uint8_t)bits;
                if (bits != 0 && bits != 255) {
                    sidx[(size_t)c] = (int32_t)surf.size();
                    surf.push_back((int32_t)c);
                }
            }
    // ambiguous configurations resolved against the face neighbour's raw case
    const int64_t ns = (int64_t)surf.size();
    std::vector<int32_t>& cases = g_mesh.cases;
    cases.resize((size_t)ns);
    for (int64_t i = 0; i < ns; ++i) {
        const int32_t c = surf[(size_t)i];
        int32_t cs = occ[(size_t)c];
        const int16_t* ck = check + 5 * cs;
        if (ck[0] == 1) {
            const int nx = c / (R * R) + ck[1], ny = c / R % R + ck[2], nz = c % R + ck[3];
            if (nx >= 0 && ny >= 0 && nz >= 0 && nx < R && ny < R && nz < R) {
                const int nb = occ[(size_t)cid(nx, ny, nz)];
                if (nb != 0 && nb != 255 && check[5 * nb] == 1) cs = ck[4];
            }
        }
        cases[(size_t)i] = cs;
    }
    // sign-changing grid edges in (first vertex, second vertex) order: for a
    // first vertex u the -y edge, then +z, then +x
    std::vector<int32_t>& edges = g_mesh.edges;
    for (int x = 0; x < RV; ++x)
        for (int y = 0; y < RV; ++y)
            for (int z = 0; z < RV; ++z) {
                const int64_t u = vid(x, y, z);
                const bool s = sdf[(size_t)u] < 0.0f;
                if (y >= 1 && s != (sdf[(size_t)vid(x, y - 1, z)] < 0.0f)) edges.insert(edges.end(), {(int32_t)u, (int32_t)vid(x, y - 1, z)});
                if (z < R && s != (sdf[(size_t)(u + 1)] < 0.0f)) edges.insert(edges.end(), {(int32_t)u, (int32_t)(u + 1)});
                if (x < R && s != (sdf[(size_t)vid(x + 1, y, z)] < 0.0f)) edges.insert(edges.end(), {(int32_t)u, (int32_t)vid(x + 1, y, z)});
            }
    // dual vertices: grouped by dual count, then surface order, then local index
    int64_t per_count[5] = {0, 0, 0, 0, 0};
    for (int64_t i = 0; i < ns; ++i) ++per_count[num_dual[cases[(size_t)i]]];
    int64_t base[5] = {0, 0, 0, 0, 0};
    for (int k = 1; k < 5; ++k) base[k] = base[k - 1] + per_count[k - 1] * (k - 1);
    const int64_t nd_total = base[4] + per_count[4] * 4;
    g_mesh.vertices.assign((size_t)nd_total * 3, 0.0f);
    g_mesh.attrs.assign((size_t)nd_total * 6, 0.0f);
    std::vector<float> dual_gamma((size_t)nd_total);
    std::vector<int32_t> dmap((size_t)ns * 12, 0);
    int64_t rank[5] = {0, 0, 0, 0, 0};
    for (int64_t i = 0; i < ns; ++i) {
        const int32_t c = surf[(size_t)i];
        const int cs = cases[(size_t)i];
        const int nd = num_dual[cs];
        const int cx = c / (R * R), cy = c / R % R, cz = c % R;
        int64_t vtx[8];
        for (int k = 0; k < 8; ++k) vtx[k] = vid(cx + kCorner[k][0], cy + kCorner[k][1], cz + kCorner[k][2]);
        const int32_t row = cube_row[(size_t)c];
        const auto w = [&](int ch) { return row < 0 ? 0.0f : raw[(size_t)row * RAW + 32 + ch]; };
        float beta[12], alpha[8];
        for (int e = 0; e < 12; ++e) beta[e] = std::tanh(w(e)) * 0.99f + 1.0f;
        for (int k = 0; k < 8; ++k) alpha[k] = std::tanh(w(12 + k)) * 0.99f + 1.0f;
        const float gamma = 1.0f / (1.0f + std::exp(-w(20))) * 0.99f + 0.005f;
        const int64_t first_id = base[nd] + rank[nd]++ * nd;
        for (int j = 0; j < nd; ++j) {
            const int64_t id = first_id + j;
            float pos[3] = {0, 0, 0}, col[6] = {0, 0, 0, 0, 0, 0}, beta_sum = 0.0f;
            for (int t = 0; t < 7; ++t) {
                const int e = dmc[(cs * 4 + j) * 7 + t];
                if (e < 0) continue;
                const int ka = kEdge[e][0], kb = kEdge[e][1];
                const float wa = sdf[(size_t)vtx[ka]] * alpha[ka];
                const float wb = sdf[(size_t)vtx[kb]] * alpha[kb];
                const float den = wb - wa;
                float va[9], vb[9];
                vertex_attr(vtx[ka], va);
                vertex_attr(vtx[kb], vb);
                beta_sum += beta[e];
                for (int a = 0; a < 3; ++a) pos[a] += ((va[a] * wb - vb[a] * wa) / den) * beta[e];
                for (int ch = 0; ch < 6; ++ch) col[ch] += ((va[3 + ch] * wb - vb[3 + ch] * wa) / den) * beta[e];
                dmap[(size_t)i * 12 + e] = (int32_t)id;
            }
            for (int a = 0; a < 3; ++a) g_mesh.vertices[(size_t)id * 3 + a] = pos[a] / beta_sum;
            for (int ch = 0; ch < 6; ++ch) g_mesh.attrs[(size_t)id * 6 + ch] = col[ch] / beta_sum;
            dual_gamma[(size_t)id] = gamma;
        }
    }
    // one quad per surface edge with four incident cubes; flipped quads first
    std::vector<int32_t> flipped, straight;
    const int64_t ne = (int64_t)edges.size() / 2;
    for (int64_t s = 0; s < ne; ++s) {
        const int64_t u = edges[(size_t)s * 2], v = edges[(size_t)s * 2 + 1];
        const int ux = (int)(u / ((int64_t)RV * RV)), uy = (int)(u / RV % RV), uz = (int)(u % RV);
        int64_t cubes[4];
        int m = 0;
        for (int d0 = 0; d0 < 2; ++d0)
            for (int d1 = 0; d1 < 2; ++d1) {
                int x = ux, y = uy, z = uz;
                if (v == u + (int64_t)RV * RV) y -= d0, z -= d1;       // +x edge
                else if (v == u + 1) x -= d0, y -= d1;                 // +z edge
                else x -= d0, y -= 1, z -= d1;                         // -y edge
                if (x < 0 || y < 0 || z < 0 || x >= R || y >= R || z >= R) continue;
                cubes[m++] = cid(x, y, z);
            }
        if (m != 4) continue;
        std::sort(cubes, cubes + 4);
        int32_t q[4];
        for (int j = 0; j < 4; ++j) {
            const int64_t c = cubes[j];
            const int cx = (int)(c / (R * R)), cy = (int)(c / R % R), cz = (int)(c % R);
            int e = 0;
            for (; e < 12; ++e) {
                const int ka = kEdge[e][0], kb = kEdge[e][1];
                if (vid(cx + kCorner[ka][0], cy + kCorner[ka][1], cz + kCorner[ka][2]) == u &&
                    vid(cx + kCorner[kb][0], cy + kCorner[kb][1], cz + kCorner[kb][2]) == v)
                    break;
            }
            q[j] = dmap[(size_t)sidx[(size_t)c] * 12 + e];
        }
        const bool flip = sdf[(size_t)u] > 0.0f;
        const int32_t o[4] = {flip ? q[0] : q[2], flip ? q[1] : q[3], flip ? q[3] : q[1], flip ? q[2] : q[0]};
        const bool split1 = dual_gamma[(size_t)o[0]] * dual_gamma[(size_t)o[2]] > dual_gamma[(size_t)o[1]] * dual_gamma[(size_t)o[3]];
        std::vector<int32_t>& dst = flip ? flipped : straight;
        if (split1) dst.insert(dst.end(), {o[0], o[1], o[2], o[0], o[2], o[3]});
        else dst.insert(dst.end(), {o[0], o[1], o[3], o[3], o[1], o[2]});
    }
    g_mesh.faces = std::move(flipped);
    g_mesh.faces.insert(g_mesh.faces.end(), straight.begin(), straight.end());
    if (counts) {
        counts[0] = nd_total;
        counts[1] = (int64_t)g_mesh.faces.size() / 3;
        counts[2] = ns;
        counts[3] = ne;
    }
    return 0;
}

// Copies the last oracle_flexicubes result; any pointer may be NULL.
void oracle_flexicubes_fetch(float* vertices, float* attrs, int32_t* faces, int32_t* surface, int32_t* cases,
                             int32_t* edges) {
    using fcx::g_mesh;
    const auto put = [](auto* dst, const auto& v) {
        if (dst && !v.empty()) std::memcpy(dst, v.data(), v.size() * sizeof(v[0]));
    };
    put(vertices, g_mesh.vertices);
    put(attrs, g_mesh.attrs);
    put(faces, g_mesh.faces);
    put(surface, g_mesh.surface);
    put(cases, g_mesh.cases);
    put(edges, g_mesh.edges);
}

}  // extern "C"
