// graph_build.cpp -- host-side restatement of GraphGP.jl's build_graph (the input producer of
// the refine path).  The refine kernels consume the graph this builds; the build itself is not
// accelerated (it is the reference's CPU algorithm, reproduced so that its output is
// byte-identical: same neighbours, offsets and permutation).
//
// Steps, each following the reference function named:
//   1. heap-order ("special order") k-d tree    src/tree_special.jl:165-227 (build_tree_special)
//   2. preceding k-NN, stackless traversal       src/tree_special.jl:231-332
//   3. longest-path depth per point              src/graph_build.jl:78-107
//   4. stable re-sort by depth + neighbour remap src/graph_build.jl:160-200
//   5. 21-bit lattice quantisation               src/graph_build.jl:231-242
//   6. batch offsets                             src/graph_build.jl:213-222
//
// The per-level sort of step 1 orders points by (node id, coordinate along the node's split
// dimension, current position): a total order, so any correct sort yields the same permutation.
// Points of one node are contiguous after the previous level's relabel, so the sort is done per
// node segment (independent, parallel) and the segments are then placed in node-id order.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <new>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

#include "gpb2_internal.h"

namespace {

inline int flevel(int64_t x) {  // floor(log2(x)) for x >= 1
    return 63 - __builtin_clzll((unsigned long long)x);
}
inline int64_t sp_parent(int64_t c) {
    if (c == 0) return -1;
    int level = flevel(c + 1);
    int64_t n_above = (int64_t(1) << level) - 1;
    int64_t n_parent_level = int64_t(1) << (level - 1);
    return c < n_above + n_parent_level ? c - n_parent_level : c - 2 * n_parent_level;
}
inline int64_t sp_left(int64_t c) { return c + (int64_t(1) << flevel(c + 1)); }
inline int64_t sp_right(int64_t c) { return c + 2 * (int64_t(1) << flevel(c + 1)); }

// Merge-sort helper for large segments: sort `nch` chunks in parallel, then merge pairwise.
template <class Cmp>
void parallel_sort(int64_t* a, int64_t n, int64_t* scratch, Cmp cmp, int nt) {
    if (nt <= 1 || n < (int64_t(1) << 16)) {
        std::sort(a, a + n, cmp);
        return;
    }
    int nch = 1;
    while (nch * 2 <= nt && (n / (nch * 2)) >= 4096) nch *= 2;
    std::vector<int64_t> bnd(nch + 1);
    for (int c = 0; c <= nch; c++) bnd[c] = n * c / nch;
#pragma omp parallel for schedule(static, 1) num_threads(nt)
    for (int c = 0; c < nch; c++) std::sort(a + bnd[c], a + bnd[c + 1], cmp);
    int64_t* src = a;
    int64_t* dst = scratch;
    int width = 1;
    while (width < nch) {
        int npairs = nch / (2 * width);
#pragma omp parallel for schedule(static, 1) num_threads(nt)
        for (int pr = 0; pr < npairs; pr++) {
            int64_t lo = bnd[2 * pr * width], mid = bnd[(2 * pr + 1) * width],
                    hi = bnd[(2 * pr + 2) * width];
            std::merge(src + lo, src + mid, src + mid, src + hi, dst + lo, cmp);
        }
        std::swap(src, dst);
        width *= 2;
    }
    if (src != a) std::memcpy(a, src, sizeof(int64_t) * n);
}

struct Tree {
    std::vector<double> pts;      // (N, D) point-major, tree order
    std::vector<int> split_dims;  // node-id indexed, 0-based dims
    std::vector<int64_t> perm;    // perm[tree_pos] = original index (0-based)
};

// src/tree_special.jl:165-227.
void build_tree_special(const double* pts_in /*(N,D) point-major*/, int64_t N, int D, int nt,
                        Tree& out) {
    int n_levels = N > 0 ? flevel(N) + 1 : 0;
    std::vector<double> pts(pts_in, pts_in + N * D), pts_s(N * D);
    std::vector<int64_t> nodes(N, 0), nodes_s(N), indices(N), indices_s(N);
    for (int64_t i = 0; i < N; i++) indices[i] = i;
    std::vector<int> split_dims(N, -1);
    std::vector<double> pad(N);
    std::vector<int64_t> p(N), p_s(N);

    for (int level = 0; level < n_levels; level++) {
        int64_t n_above = (int64_t(1) << level) - 1;
        int64_t n_level = int64_t(1) << level;

        // Segments: after the previous relabel every node's points are one contiguous run.
        // Collect runs (start, node) in position order.
        std::vector<int64_t> run_start;
        run_start.reserve(std::min<int64_t>(N, 2 * n_level + n_above + 2));
        for (int64_t i = 0; i < N; i++)
            if (i == 0 || nodes[i] != nodes[i - 1]) run_start.push_back(i);
        int64_t nruns = (int64_t)run_start.size();
        run_start.push_back(N);

        // Split dimension of every node id >= n_above: widest extent of its points
        // (src/tree_special.jl:41-65).  Node ids without points get dim 0 (range -Inf).
#pragma omp parallel for schedule(static) num_threads(nt)
        for (int64_t i = n_above; i < N; i++) split_dims[i] = 0;
#pragma omp parallel for schedule(dynamic, 64) num_threads(nt)
        for (int64_t r = 0; r < nruns; r++) {
            int64_t s = nodes[run_start[r]];
            if (s < n_above) continue;
            double mx[8], mn[8];
            for (int d = 0; d < D; d++) {
                mx[d] = -std::numeric_limits<double>::infinity();
                mn[d] = std::numeric_limits<double>::infinity();
            }
            for (int64_t i = run_start[r]; i < run_start[r + 1]; i++)
                for (int d = 0; d < D; d++) {
                    double v = pts[i * D + d];
                    if (v > mx[d]) mx[d] = v;
                    if (v < mn[d]) mn[d] = v;
                }
            int bestd = 0;
            double bestr = -std::numeric_limits<double>::infinity();
            for (int d = 0; d < D; d++) {
                double rr = mx[d] - mn[d];
                if (rr > bestr) { bestr = rr; bestd = d; }
            }
            if (s < N) split_dims[s] = bestd;
        }
#pragma omp parallel for schedule(static) num_threads(nt)
        for (int64_t i = 0; i < N; i++) {
            int64_t s = nodes[i];
            pad[i] = pts[i * D + split_dims[s < N ? s : 0]];
        }
        // Runs in node-id order; each run sorted by (pad, position).
        std::vector<int64_t> order(nruns);
        for (int64_t r = 0; r < nruns; r++) order[r] = r;
        std::sort(order.begin(), order.end(), [&](int64_t a, int64_t b) {
            return nodes[run_start[a]] < nodes[run_start[b]];
        });
        std::vector<int64_t> dst_start(nruns);
        {
            int64_t acc = 0;
            for (int64_t t = 0; t < nruns; t++) {
                int64_t r = order[t];
                dst_start[r] = acc;
                acc += run_start[r + 1] - run_start[r];
            }
        }
        auto cmp = [&](int64_t a, int64_t b) {
            double pa = pad[a], pb = pad[b];
            if (pa != pb) return pa < pb;
            return a < b;
        };
        // Large runs: parallel sort inside; small runs: one thread each.
        const int64_t big = int64_t(1) << 18;
        for (int64_t r = 0; r < nruns; r++) {
            int64_t len = run_start[r + 1] - run_start[r];
            if (len < big) continue;
            int64_t* seg = p.data() + dst_start[r];
            for (int64_t i = 0; i < len; i++) seg[i] = run_start[r] + i;
            parallel_sort(seg, len, p_s.data() + dst_start[r], cmp, nt);
        }
#pragma omp parallel for schedule(dynamic, 16) num_threads(nt)
        for (int64_t r = 0; r < nruns; r++) {
            int64_t len = run_start[r + 1] - run_start[r];
            if (len >= big) continue;
            int64_t* seg = p.data() + dst_start[r];
            for (int64_t i = 0; i < len; i++) seg[i] = run_start[r] + i;
            std::sort(seg, seg + len, cmp);
        }
        // Gather (src/tree_special.jl:74-85).
#pragma omp parallel for schedule(static) num_threads(nt)
        for (int64_t i = 0; i < N; i++) {
            int64_t pp = p[i];
            for (int d = 0; d < D; d++) pts_s[i * D + d] = pts[pp * D + d];
            nodes_s[i] = nodes[pp];
            indices_s[i] = indices[pp];
        }
        pts.swap(pts_s);
        indices.swap(indices_s);
        nodes.swap(nodes_s);
        // Relabel: even-by-id redistribution (src/tree_special.jl:87-99).
        int64_t n_remaining = N - n_above;
        int64_t q = n_remaining / n_level;
        int64_t rr = n_remaining % n_level;
#pragma omp parallel for schedule(static) num_threads(nt)
        for (int64_t idx = 0; idx < N; idx++) {
            int64_t s = nodes[idx];
            int64_t ii = s - n_above;
            int64_t mid = (ii < rr ? ii * (q + 1) + (q + 1) / 2
                                   : rr * (q + 1) + (ii - rr) * q + q / 2) + n_above;
            nodes_s[idx] = (idx < n_above || idx == mid) ? s
                           : (idx < mid ? s + n_level : s + 2 * n_level);
        }
        nodes.swap(nodes_s);
    }
    out.pts.swap(pts);
    out.split_dims.swap(split_dims);
    out.perm.swap(indices);
}

// src/tree_special.jl:231-293: exact stackless traversal for one query node.
void query_one(double* cand_d, int64_t* cand_i, const double* sp, const int* split_dims,
               int64_t query, int64_t max_index, int k, int D) {
    for (int j = 0; j < k; j++) {
        cand_d[j] = std::numeric_limits<double>::infinity();
        cand_i[j] = -1;
    }
    double square_radius = std::numeric_limits<double>::infinity();
    const double* q = sp + query * D;
    int64_t current = 0, previous = -1;
    while (current != -1) {
        int64_t parent = sp_parent(current);
        if (previous == parent) {
            const double* c = sp + current * D;
            double sq = 0.0;
            for (int d = 0; d < D; d++) {
                double dv = q[d] - c[d];
                sq += dv * dv;
            }
            int wpos = 0;
            double wval = cand_d[0];
            for (int j = 1; j < k; j++)
                if (cand_d[j] > wval) { wval = cand_d[j]; wpos = j; }
            if (sq < wval) {
                cand_d[wpos] = sq;
                cand_i[wpos] = current;
                double m = cand_d[0];
                for (int j = 1; j < k; j++)
                    if (cand_d[j] > m) m = cand_d[j];
                square_radius = m;
            } else {
                square_radius = wval;
            }
        }
        int sd = split_dims[current];
        double split_distance = q[sd] - sp[current * D + sd];
        int64_t near = split_distance < 0 ? sp_left(current) : sp_right(current);
        int64_t far = split_distance < 0 ? sp_right(current) : sp_left(current);
        bool far_in_range = split_distance * split_distance <= square_radius;
        int64_t nxt;
        if (previous == near || (previous == parent && near >= max_index))
            nxt = (far < max_index && far_in_range) ? far : parent;
        else
            nxt = previous == parent ? near : parent;
        previous = current;
        current = nxt;
    }
}

}  // namespace

struct gpb2_graph {
    int64_t n = 0, d = 0, n0 = 0, k = 0;
    double scale = 0.0;
    std::vector<uint32_t> coords;   // (N, D) point-major, depth order
    std::vector<int64_t> nbrs;      // (M, K) point-major, 0-based, -1 = unset
    std::vector<int64_t> indices;   // tree position -> original index (0-based)
    std::vector<int64_t> offsets;   // offsets[0] = n0, last = N
};

extern "C" {

int gpb2_build_graph(const double* points, int64_t n, int64_t d, int64_t points_dim_major,
                     int64_t n0, int64_t k, int64_t lattice_bits, int64_t nthreads,
                     gpb2_graph** out) {
    using namespace gpb2;
    if (!out) return set_error(GPB2_ERR_INVALID_ARG, "gpb2_build_graph: out is NULL");
    *out = nullptr;
    if (!points || n <= 0 || d < 1 || d > 8 || k < 1 || k > 64 || n0 < 1 || n0 >= n ||
        lattice_bits < 1 || lattice_bits > 31)
        return set_error(GPB2_ERR_INVALID_ARG,
                         "gpb2_build_graph: need points, 1<=d<=8, 1<=k<=64, 1<=n0<n, "
                         "1<=lattice_bits<=31 (got n=%lld d=%lld n0=%lld k=%lld bits=%lld)",
                         (long long)n, (long long)d, (long long)n0, (long long)k,
                         (long long)lattice_bits);
    int nt = 1;
#ifdef _OPENMP
    nt = nthreads > 0 ? (int)nthreads : omp_get_max_threads();
#endif
    const int D = (int)d;
    const int K = (int)k;
    try {
        std::vector<double> pm((size_t)(n * d));
        if (points_dim_major) {
#pragma omp parallel for schedule(static) num_threads(nt)
            for (int64_t i = 0; i < n; i++)
                for (int dd = 0; dd < D; dd++) pm[i * D + dd] = points[dd * n + i];
        } else {
            std::memcpy(pm.data(), points, sizeof(double) * n * d);
        }
        Tree tree;
        build_tree_special(pm.data(), n, D, nt, tree);
        std::vector<double>().swap(pm);

        // Step 2: preceding k-NN, each column sorted by (distance, index).
        const int64_t M = n - n0;
        std::vector<int64_t> nb((size_t)(M * K));
#pragma omp parallel num_threads(nt)
        {
            std::vector<double> cd(K);
            std::vector<int64_t> ci(K), ord(K);
#pragma omp for schedule(dynamic, 256)
            for (int64_t m = n0; m < n; m++) {
                query_one(cd.data(), ci.data(), tree.pts.data(), tree.split_dims.data(), m, m, K,
                          D);
                for (int j = 0; j < K; j++) ord[j] = j;
                std::sort(ord.begin(), ord.end(), [&](int64_t a, int64_t b) {
                    if (cd[a] != cd[b]) return cd[a] < cd[b];
                    return ci[a] < ci[b];
                });
                for (int j = 0; j < K; j++) nb[(m - n0) * K + j] = ci[ord[j]];
            }
        }

        // Step 3: depths (one in-order pass reaches the fixed point: neighbours precede).
        std::vector<int64_t> depth((size_t)n, 0);
        for (int64_t m = 0; m < M; m++) {
            int64_t mx = 0;
            for (int j = 0; j < K; j++) {
                int64_t v = nb[m * K + j];
                if (v < 0) continue;
                if (depth[v] > mx) mx = depth[v];
            }
            depth[n0 + m] = mx + 1;
        }

        // Step 4: stable sort by depth (counting sort), remap neighbours.
        int64_t maxd = 0;
        for (int64_t i = 0; i < n; i++) maxd = std::max(maxd, depth[i]);
        std::vector<int64_t> cnt((size_t)maxd + 2, 0);
        for (int64_t i = 0; i < n; i++) cnt[depth[i] + 1]++;
        for (int64_t dd = 0; dd <= maxd; dd++) cnt[dd + 1] += cnt[dd];
        std::vector<int64_t> sort_perm((size_t)n), inv_sp((size_t)n);
        {
            std::vector<int64_t> pos(cnt.begin(), cnt.end() - 1);
            for (int64_t i = 0; i < n; i++) sort_perm[pos[depth[i]]++] = i;
        }
        for (int64_t i = 0; i < n; i++) inv_sp[sort_perm[i]] = i;
        int64_t n0_new = cnt[1];

        auto* g = new gpb2_graph();
        g->n = n;
        g->d = d;
        g->k = k;
        g->n0 = n0_new;
        g->indices.resize((size_t)n);
        for (int64_t i = 0; i < n; i++) g->indices[i] = tree.perm[sort_perm[i]];
        g->nbrs.assign((size_t)((n - n0_new) * K), -1);
        for (int64_t m_old = 0; m_old < M; m_old++) {
            int64_t m_new = inv_sp[n0 + m_old] - n0_new;
            if (m_new < 0) continue;
            for (int j = 0; j < K; j++) {
                int64_t old_nb = nb[m_old * K + j];
                if (old_nb < 0) continue;
                g->nbrs[m_new * K + j] = inv_sp[old_nb];
            }
        }
        std::vector<int64_t>().swap(nb);

        // Step 5: quantise the depth-ordered points (src/graph_build.jl:231-242).
        const double lmax = double((int64_t(1) << lattice_bits) - 1);
        std::vector<double> origin(D, std::numeric_limits<double>::infinity()),
            hi(D, -std::numeric_limits<double>::infinity());
        for (int64_t i = 0; i < n; i++)
            for (int dd = 0; dd < D; dd++) {
                double v = tree.pts[i * D + dd];
                origin[dd] = std::min(origin[dd], v);
                hi[dd] = std::max(hi[dd], v);
            }
        double extent = -std::numeric_limits<double>::infinity();
        for (int dd = 0; dd < D; dd++) extent = std::max(extent, hi[dd] - origin[dd]);
        double scale = extent > 0 ? extent / lmax : 1.0 / lmax;
        g->scale = scale;
        g->coords.resize((size_t)(n * d));
#pragma omp parallel for schedule(static) num_threads(nt)
        for (int64_t i = 0; i < n; i++) {
            int64_t src = sort_perm[i];
            for (int dd = 0; dd < D; dd++) {
                double cf = (tree.pts[src * D + dd] - origin[dd]) / scale;
                double rnd = std::nearbyint(cf);  // round half to even (default mode)
                int64_t c = (int64_t)rnd;
                if (c < 0) c = 0;
                if (c > (int64_t)lmax) c = (int64_t)lmax;
                g->coords[i * D + dd] = (uint32_t)c;
            }
        }
        // Step 6: offsets[d] = number of points with depth <= d.
        g->offsets.resize((size_t)maxd + 1);
        for (int64_t dd = 0; dd <= maxd; dd++) g->offsets[dd] = cnt[dd + 1];
        *out = g;
    } catch (const std::bad_alloc&) {
        return set_error(GPB2_ERR_OOM, "gpb2_build_graph: host allocation failed (n=%lld)",
                         (long long)n);
    }
    return GPB2_OK;
}

int64_t gpb2_graph_n_offsets(const gpb2_graph* g) { return g ? (int64_t)g->offsets.size() : -1; }
int64_t gpb2_graph_n0(const gpb2_graph* g) { return g ? g->n0 : -1; }

int gpb2_graph_export(const gpb2_graph* g, uint32_t* coords, int64_t* nbrs, int64_t* indices,
                      int64_t* offsets, double* scale) {
    using namespace gpb2;
    if (!g) return set_error(GPB2_ERR_INVALID_ARG, "gpb2_graph_export: graph is NULL");
    if (coords) std::memcpy(coords, g->coords.data(), sizeof(uint32_t) * g->coords.size());
    if (nbrs) std::memcpy(nbrs, g->nbrs.data(), sizeof(int64_t) * g->nbrs.size());
    if (indices) std::memcpy(indices, g->indices.data(), sizeof(int64_t) * g->indices.size());
    if (offsets) std::memcpy(offsets, g->offsets.data(), sizeof(int64_t) * g->offsets.size());
    if (scale) *scale = g->scale;
    return GPB2_OK;
}

void gpb2_graph_free(gpb2_graph* g) { delete g; }

}  // extern "C"
