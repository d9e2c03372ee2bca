// vt_voronoi.cu -- Voronoi face adjacency (= Delaunay neighbours) on the GPU.
//
// The reference delegates this to the external `paragram` package
// (vorotracing/cuda/__init__.py:16-46, called every 1-100 training steps,
// vorotracing/trainer.py:354-360).  Method: each site's Voronoi cell is built
// independently by clipping:
//   1. the cell starts as a box around the site (16x the scene extent) and is
//      clipped by the bisector planes of nearby sites (seeds);
//   2. every vertex v of the cell is then verified by the empty-ball
//      property of Delaunay: no site may be closer to v than the cell's own
//      site.  The ball B(v, |v - p_i|) is searched in a BVH of the sites; a
//      site found inside it clips the cell (removing v) and verification
//      continues over the new vertices until every ball is empty;
//   3. the neighbours whose planes still bound the cell are the site's
//      Voronoi neighbours.
// The verified cell is the exact Voronoi cell (within the box), however
// elongated: cells of sites on dense sheets are long needles whose bounding
// sites are far away, and the ball search touches only the BVH nodes those
// needles' vertex balls reach.  Cells of convex-hull sites are unbounded and
// come out as their intersection with the box, so a face lying entirely
// beyond the box is missing.
// The first pass builds one cell per warp in shared memory
// (vt_voronoi_warp.cuh); the cells it cannot finish are rebuilt here one per
// thread (cell_verify_kernel: 48 exact nearest-site seeds, the cell in local
// memory), then, if that fails too, by clipping with every site ring by ring
// around the site (cell_stream_kernel, up to 16384).
// The cell is stored in dual form: each vertex is a triangle of three plane
// ids (counter-clockwise seen from outside) with its position and the three
// neighbouring triangles across its edges.  A clip removes the triangles
// whose vertex lies beyond the plane and closes the hole with a fan of new
// triangles around the new plane.  Coordinates are relative to the site, so
// bisector planes are n.x = |n|^2 / 2 with n = p_j - p_i.  Predicates are
// binary32, so a near-degenerate clip sequence can fail; the later passes
// clip in another order.
#include <cub/device/device_scan.cuh>

#include "vt_abi.cuh"
#include "vt_bvh.cuh"

namespace vt {
namespace vor {

constexpr int kMaxPlanes = 128;  // 6 box planes + clipping planes kept
constexpr int kMaxTris = 254;    // cell vertices (uint8 ids, 255 = none)
constexpr int kMaxRing = 128;    // boundary edges of one clip
constexpr uint8_t kNone = 0xff;

struct Cell {
    float4 plane[kMaxPlanes];      // n.xyz, d : n.x <= d inside
    uint32_t site[kMaxPlanes];     // neighbour id, 0xffffffff for box planes
    uint8_t tri[kMaxTris][3];      // plane ids
    uint8_t nbr[kMaxTris][3];      // triangle across edge (v0v1, v1v2, v2v0)
    float3 pos[kMaxTris];
    uint8_t alive[kMaxTris];       // 0 removed, 1 live, 2 live and verified (empty ball)
    int nplanes, ntris;
};

__device__ __forceinline__ bool solve3(float4 a, float4 b, float4 c, float3 &x)
{
    // Cramer's rule for [a;b;c] x = d
    float3 bc = make_float3(b.y * c.z - b.z * c.y, b.z * c.x - b.x * c.z, b.x * c.y - b.y * c.x);
    float det = a.x * bc.x + a.y * bc.y + a.z * bc.z;
    if (fabsf(det) < 1e-30f) return false;
    float3 ca = make_float3(c.y * a.z - c.z * a.y, c.z * a.x - c.x * a.z, c.x * a.y - c.y * a.x);
    float3 ab = make_float3(a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x);
    float inv = 1.0f / det;
    x = make_float3((a.w * bc.x + b.w * ca.x + c.w * ab.x) * inv,
                    (a.w * bc.y + b.w * ca.y + c.w * ab.y) * inv,
                    (a.w * bc.z + b.w * ca.z + c.w * ab.z) * inv);
    return true;
}

__device__ void init_box(Cell &C, float B)
{
    // planes 0..5: +x, -x, +y, -y, +z, -z
    const float4 P[6] = {{1, 0, 0, B}, {-1, 0, 0, B}, {0, 1, 0, B},
                         {0, -1, 0, B}, {0, 0, 1, B}, {0, 0, -1, B}};
    for (int i = 0; i < 6; ++i) {
        C.plane[i] = P[i];
        C.site[i] = 0xffffffffu;
    }
    C.nplanes = 6;
    // 8 corners as triangles of three planes, consistently oriented
    const uint8_t T[8][3] = {{0, 2, 4}, {0, 5, 2}, {0, 3, 5}, {0, 4, 3},
                             {1, 4, 2}, {1, 2, 5}, {1, 5, 3}, {1, 3, 4}};
    for (int t = 0; t < 8; ++t) {
        for (int k = 0; k < 3; ++k) C.tri[t][k] = T[t][k];
        float3 x;
        solve3(C.plane[T[t][0]], C.plane[T[t][1]], C.plane[T[t][2]], x);
        C.pos[t] = x;
        C.alive[t] = 1;
    }
    C.ntris = 8;
    // neighbours: the triangle sharing the reversed edge
    for (int t = 0; t < 8; ++t)
        for (int k = 0; k < 3; ++k) {
            uint8_t a = C.tri[t][k], b = C.tri[t][(k + 1) % 3];
            C.nbr[t][k] = kNone;
            for (int u = 0; u < 8; ++u)
                for (int m = 0; m < 3; ++m)
                    if (C.tri[u][m] == b && C.tri[u][(m + 1) % 3] == a) C.nbr[t][k] = (uint8_t)u;
        }
}

// Drop planes no live triangle uses (renumbering the rest), to make room.
__device__ void compact_planes(Cell &C)
{
    uint8_t remap[kMaxPlanes];
    bool used[kMaxPlanes];
    for (int p = 0; p < C.nplanes; ++p) used[p] = p < 6;
    for (int t = 0; t < C.ntris; ++t)
        if (C.alive[t])
            for (int m = 0; m < 3; ++m) used[C.tri[t][m]] = true;
    int k = 0;
    for (int p = 0; p < C.nplanes; ++p) {
        remap[p] = (uint8_t)k;
        if (used[p]) {
            C.plane[k] = C.plane[p];
            C.site[k] = C.site[p];
            ++k;
        }
    }
    for (int t = 0; t < C.ntris; ++t)
        if (C.alive[t])
            for (int m = 0; m < 3; ++m) C.tri[t][m] = remap[C.tri[t][m]];
    C.nplanes = k;
}

// Clip by plane (n, d).  Returns false on overflow / degeneracy (cell
// unusable); *cut (if given) tells whether the plane removed any vertex.
__device__ bool clip(Cell &C, float4 pl, uint32_t site, bool *cut = nullptr)
{
    bool out[kMaxTris];
    int nout = 0, nin = 0;
    for (int t = 0; t < C.ntris; ++t) {
        out[t] = false;
        if (!C.alive[t]) continue;
        float3 p = C.pos[t];
        if (pl.x * p.x + pl.y * p.y + pl.z * p.z - pl.w > 0.0f) {
            out[t] = true;
            ++nout;
        } else {
            ++nin;
        }
    }
    if (cut) *cut = nout > 0;
    if (nout == 0) return true;  // plane misses the cell
    if (nin == 0) return false;  // everything cut: degenerate input
    if (C.nplanes >= kMaxPlanes) compact_planes(C);
    if (C.nplanes >= kMaxPlanes) return false;
    const int np = C.nplanes;
    // boundary edges a->b of removed triangles whose neighbour survives
    uint8_t ea[kMaxRing], eb[kMaxRing], en[kMaxRing];
    int ne = 0;
    for (int t = 0; t < C.ntris; ++t) {
        if (!out[t]) continue;
        for (int k = 0; k < 3; ++k) {
            uint8_t n = C.nbr[t][k];
            if (n == kNone) return false;
            if (out[n]) continue;
            if (ne >= kMaxRing) return false;
            ea[ne] = C.tri[t][k];
            eb[ne] = C.tri[t][(k + 1) % 3];
            en[ne] = n;
            ++ne;
        }
    }
    if (ne < 3) return false;
    for (int t = 0; t < C.ntris; ++t)
        if (out[t]) C.alive[t] = 0;
    C.plane[np] = pl;
    C.site[np] = site;
    int8_t start_of[kMaxPlanes];
    for (int i = 0; i <= np; ++i) start_of[i] = -1;
    uint8_t slot_of[kMaxRing];
    int scan = 0;
    for (int e = 0; e < ne; ++e) {
        while (scan < C.ntris && C.alive[scan]) ++scan;
        int slot;
        if (scan < C.ntris) {
            slot = scan++;
        } else {
            if (C.ntris >= kMaxTris) return false;
            slot = C.ntris++;
            scan = C.ntris;
        }
        const uint8_t a = ea[e], b = eb[e], n = en[e];
        float3 x;
        if (!solve3(C.plane[a], C.plane[b], pl, x)) return false;
        C.tri[slot][0] = a;
        C.tri[slot][1] = b;
        C.tri[slot][2] = (uint8_t)np;
        C.nbr[slot][0] = n;
        C.nbr[slot][1] = kNone;
        C.nbr[slot][2] = kNone;
        C.pos[slot] = x;
        C.alive[slot] = 1;
        for (int m = 0; m < 3; ++m)
            if (C.tri[n][m] == b && C.tri[n][(m + 1) % 3] == a) C.nbr[n][m] = (uint8_t)slot;
        if (start_of[a] != -1) return false;  // boundary is not a simple cycle
        start_of[a] = (int8_t)e;
        slot_of[e] = (uint8_t)slot;
    }
    // fan around the new plane: (a, b, np) is followed by the triangle whose
    // boundary edge starts at b
    for (int e = 0; e < ne; ++e) {
        int f = start_of[eb[e]];
        if (f < 0) return false;
        C.nbr[slot_of[e]][1] = slot_of[f];
        C.nbr[slot_of[f]][2] = slot_of[e];
    }
    C.nplanes = np + 1;
    return true;
}

__device__ float max_vertex_r2(const Cell &C)
{
    float r2 = 0.0f;
    for (int t = 0; t < C.ntris; ++t)
        if (C.alive[t]) {
            float3 v = C.pos[t];
            r2 = fmaxf(r2, v.x * v.x + v.y * v.y + v.z * v.z);
        }
    return r2;
}

// Neighbour ids of the planes that still bound the cell, ascending.
__device__ uint32_t emit(const Cell &C, uint32_t *out, uint32_t stride)
{
    bool used[kMaxPlanes];
    for (int p = 0; p < C.nplanes; ++p) used[p] = false;
    for (int t = 0; t < C.ntris; ++t)
        if (C.alive[t])
            for (int m = 0; m < 3; ++m) used[C.tri[t][m]] = true;
    uint32_t c = 0;
    for (int p = 6; p < C.nplanes; ++p)
        if (used[p] && c < stride) out[c++] = C.site[p];
    for (uint32_t a = 1; a < c; ++a) {
        uint32_t v = out[a];
        uint32_t b = a;
        while (b > 0 && out[b - 1] > v) {
            out[b] = out[b - 1];
            --b;
        }
        out[b] = v;
    }
    return c;
}

}  // namespace vor
}  // namespace vt

namespace vt {
namespace vor {

struct Grid {
    float3 lo;
    float inv_h;
    int3 dim;
};

__device__ __forceinline__ int3 cell_of(const Grid &g, float3 p)
{
    int3 c;
    c.x = min(max((int)((p.x - g.lo.x) * g.inv_h), 0), g.dim.x - 1);
    c.y = min(max((int)((p.y - g.lo.y) * g.inv_h), 0), g.dim.y - 1);
    c.z = min(max((int)((p.z - g.lo.z) * g.inv_h), 0), g.dim.z - 1);
    return c;
}

__global__ void grid_count(const float *__restrict__ p, uint32_t n, Grid g, uint32_t *cnt,
                           uint32_t *cell_id)
{
    uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    int3 c = cell_of(g, make_float3(p[3 * i], p[3 * i + 1], p[3 * i + 2]));
    uint32_t id = ((uint32_t)c.z * g.dim.y + c.y) * g.dim.x + c.x;
    cell_id[i] = id;
    atomicAdd(cnt + id, 1u);
}

__global__ void grid_scatter(uint32_t n, const uint32_t *cell_id, uint32_t *cursor, uint32_t *sorted)
{
    uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint32_t slot = atomicAdd(cursor + cell_id[i], 1u);
    sorted[slot] = i;
}

// Sites of each grid cell in ascending id order (the scatter's atomic slots
// are in arbitrary order), so that every scan order is reproducible.
__global__ void grid_sort(uint32_t ncells, const uint32_t *__restrict__ start, uint32_t *sorted)
{
    const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= ncells) return;
    const uint32_t b = start[c], e = start[c + 1];
    for (uint32_t a = b + 1; a < e; ++a) {
        const uint32_t v = sorted[a];
        uint32_t k = a;
        while (k > b && sorted[k - 1] > v) {
            sorted[k] = sorted[k - 1];
            --k;
        }
        sorted[k] = v;
    }
}

// k nearest neighbours of site i (excluding i), ascending (distance, id).
__device__ int knn(const float *__restrict__ p, uint32_t i, const Grid &g,
                   const uint32_t *__restrict__ start, const uint32_t *__restrict__ sorted, int k,
                   float *kd, uint32_t *ki)
{
    float3 q = make_float3(p[3 * i], p[3 * i + 1], p[3 * i + 2]);
    int3 c = cell_of(g, q);
    int found = 0;
    const int rmax = max(g.dim.x, max(g.dim.y, g.dim.z));
    for (int r = 0; r <= rmax; ++r) {
        // every point outside the rings scanned so far is at least (r-1) cells away
        if (found == k && r >= 1) {
            float lim = (float)(r - 1) / g.inv_h;
            if (lim * lim > kd[k - 1]) break;
        }
        for (int z = c.z - r; z <= c.z + r; ++z) {
            if (z < 0 || z >= g.dim.z) continue;
            for (int y = c.y - r; y <= c.y + r; ++y) {
                if (y < 0 || y >= g.dim.y) continue;
                for (int x = c.x - r; x <= c.x + r; ++x) {
                    if (x < 0 || x >= g.dim.x) continue;
                    if (max(abs(x - c.x), max(abs(y - c.y), abs(z - c.z))) != r) continue;
                    uint32_t id = ((uint32_t)z * g.dim.y + y) * g.dim.x + x;
                    for (uint32_t s = start[id]; s < start[id + 1]; ++s) {
                        uint32_t j = sorted[s];
                        if (j == i) continue;
                        float dx = p[3 * j] - q.x, dy = p[3 * j + 1] - q.y, dz = p[3 * j + 2] - q.z;
                        float d2 = dx * dx + dy * dy + dz * dz;
                        if (found == k && (d2 > kd[k - 1] || (d2 == kd[k - 1] && j > ki[k - 1])))
                            continue;
                        int pos = found < k ? found++ : k - 1;
                        while (pos > 0 && (kd[pos - 1] > d2 || (kd[pos - 1] == d2 && ki[pos - 1] > j))) {
                            kd[pos] = kd[pos - 1];
                            ki[pos] = ki[pos - 1];
                            --pos;
                        }
                        kd[pos] = d2;
                        ki[pos] = j;
                    }
                }
            }
        }
    }
    return found;
}

constexpr int kSeedK = 24;     // nearest sites clipped before verification
constexpr int kSeedKRetry = 48;  // the same for cells whose first clip sequence failed
constexpr int kMaxClips = 768;  // clips of one cell in verification (then the fallback)

// Clip the cell by a site that cuts its vertex v (coordinates relative to
// site i at q): a site closer to v than site i, i.e. inside the ball
// B(q + v, |v|).  The sites' BVH is traversed nearest child first, pruning
// boxes farther than |v| (with a relative slack of 2^-10 covering the
// rounding difference between absolute and site-relative coordinates); the
// cut itself is decided by the clip's own plane test.  Sites skip0..2 (the
// planes through v) are ignored.  Returns 1 if the cell was clipped, 0 if no
// site cuts v, -1 if clipping failed.
__device__ int bvh_cut(Cell &C, const float *__restrict__ p, uint32_t i, float3 q, float3 v,
                       const bvh::Node *__restrict__ nodes, const uint32_t *__restrict__ ids,
                       uint32_t skip0, uint32_t skip1, uint32_t skip2)
{
    const V3 x = mk(q.x + v.x, q.y + v.y, q.z + v.z);
    const float r2 = v.x * v.x + v.y * v.y + v.z * v.z;
    const float lim = r2 + r2 * 0.0009765625f;
    uint32_t stack[bvh::kStack];
    int sp = 0;
    uint32_t cur = 0;
    for (;;) {
        if (cur & bvh::kLeaf) {
            const uint32_t j = __ldg(ids + (cur & ~bvh::kLeaf));
            if (j != i && j != skip0 && j != skip1 && j != skip2) {
                const float nx = p[3 * j] - q.x, ny = p[3 * j + 1] - q.y, nz = p[3 * j + 2] - q.z;
                const float4 pl = make_float4(nx, ny, nz, 0.5f * (nx * nx + ny * ny + nz * nz));
                if (pl.x * v.x + pl.y * v.y + pl.z * v.z - pl.w > 0.0f) {
                    bool cut = false;
                    if (!clip(C, pl, j, &cut)) return -1;
                    if (cut) return 1;
                }
            }
        } else {
            const bvh::Node nd = nodes[cur];
            const uint32_t c[2] = {nd.left, nd.right};
            float dd[2];
            for (int k = 0; k < 2; ++k) {
                if (c[k] & bvh::kLeaf) {
                    const V3 dv = x - ld3(p + (size_t)__ldg(ids + (c[k] & ~bvh::kLeaf)) * 3);
                    dd[k] = dot(dv, dv);
                } else {
                    dd[k] = bvh::box_d2(nodes[c[k]], x);
                }
            }
            const int nearf = dd[1] < dd[0] ? 1 : 0;
            if (dd[1 - nearf] <= lim) {
                if (sp >= bvh::kStack) return -1;
                stack[sp++] = c[1 - nearf];
            }
            if (dd[nearf] <= lim) {
                cur = c[nearf];
                continue;
            }
        }
        if (sp == 0) return 0;
        cur = stack[--sp];
    }
}

// One cell per thread: clip by the kSeedK nearest sites, then verify every
// vertex v of the cell by the empty-ball property of Delaunay: no site may be
// closer to v than site i.  A site found inside a vertex's ball clips the
// cell (removing that vertex), and verification goes on over the new
// vertices until every vertex's ball is empty; the cell is then exact (for a
// convex-hull site: exact inside the truncation box).  The balls are searched
// in the sites' BVH, so long needle-shaped cells along dense sheets and far
// vertices of hull cells cost the nodes their balls touch.  Cells whose
// clipping fails (a near-degenerate clip sequence) go to the retry list; the
// retry seeds with more sites, which changes the sequence.
__global__ void __launch_bounds__(64) cell_verify_kernel(
    const float *__restrict__ p, uint32_t n, Grid g, const uint32_t *__restrict__ start,
    const uint32_t *__restrict__ sorted, const bvh::Node *__restrict__ nodes,
    const uint32_t *__restrict__ ids, float box, const uint32_t *__restrict__ todo, uint32_t ntodo,
    int seedk, const uint32_t *__restrict__ seed_adj, const uint32_t *__restrict__ seed_offs,
    uint32_t *__restrict__ nbr_out, uint32_t stride, uint32_t *__restrict__ count,
    uint32_t *__restrict__ retry, uint32_t *nretry)
{
    const uint32_t t0 = blockIdx.x * blockDim.x + threadIdx.x;
    if (t0 >= ntodo) return;
    const uint32_t i = todo ? todo[t0] : t0;
    float kd[kSeedKRetry];
    uint32_t ki[kSeedKRetry];
    int found = 0;
    if (seed_adj) {
        // the caller's guesses, nearest first (up to kSeedKRetry of them)
        const float3 qi = make_float3(p[3 * i], p[3 * i + 1], p[3 * i + 2]);
        const uint32_t b = seed_offs[i], e = seed_offs[i + 1];
        for (uint32_t k = b; k < e && found < kSeedKRetry; ++k) {
            const uint32_t j = seed_adj[k];
            if (j >= n || j == i) continue;
            const float dx = p[3 * j] - qi.x, dy = p[3 * j + 1] - qi.y, dz = p[3 * j + 2] - qi.z;
            const float d2 = dx * dx + dy * dy + dz * dz;
            int pos = found++;
            while (pos > 0 && kd[pos - 1] > d2) {
                kd[pos] = kd[pos - 1];
                ki[pos] = ki[pos - 1];
                --pos;
            }
            kd[pos] = d2;
            ki[pos] = j;
        }
    } else {
        found = knn(p, i, g, start, sorted, min(seedk, kSeedKRetry), kd, ki);
    }
    Cell C;
    init_box(C, box);
    const float3 q = make_float3(p[3 * i], p[3 * i + 1], p[3 * i + 2]);
    bool ok = true;
    for (int m = 0; m < found && ok; ++m) {
        const uint32_t j = ki[m];
        const float nx = p[3 * j] - q.x, ny = p[3 * j + 1] - q.y, nz = p[3 * j + 2] - q.z;
        ok = clip(C, make_float4(nx, ny, nz, 0.5f * (nx * nx + ny * ny + nz * nz)), j);
    }
    int clips = 0;
    int t = 0;
    while (ok && t < C.ntris) {
        if (C.alive[t] != 1) {
            ++t;
            continue;
        }
        const uint32_t s0 = C.site[C.tri[t][0]], s1 = C.site[C.tri[t][1]], s2 = C.site[C.tri[t][2]];
        const int res = bvh_cut(C, p, i, q, C.pos[t], nodes, ids, s0, s1, s2);
        if (res < 0 || ++clips > kMaxClips) {
            ok = false;
            break;
        }
        if (res == 0) {
            C.alive[t] = 2;
            ++t;
        } else {
            t = 0;  // new vertices may sit in reused slots
        }
    }
    if (!ok) {
#ifdef VT_VOR_VERBOSE
        printf("verify failed: site %u clips %d ntris %d nplanes %d\n", i, clips, C.ntris, C.nplanes);
#endif
        const uint32_t r = atomicAdd(nretry, 1u);
        retry[r] = i;
        count[i] = 0;
        return;
    }
    count[i] = emit(C, nbr_out + (size_t)i * stride, stride);
}

}  // namespace vor
}  // namespace vt

#include "vt_voronoi_warp.cuh"

namespace vt {
namespace vor {

// Final pass: clip against the sites ring by ring around the site's grid
// cell until every site not yet scanned is farther than twice the farthest
// cell vertex.  Convex-hull cells never get there (they reach the truncation
// box); they stop after kStreamCap scanned sites.
constexpr uint32_t kStreamCap = 16384;
__global__ void __launch_bounds__(64) cell_stream_kernel(
    const float *__restrict__ p, uint32_t n, Grid g, const uint32_t *__restrict__ start,
    const uint32_t *__restrict__ sorted, float box, const uint32_t *__restrict__ todo,
    uint32_t ntodo, uint32_t *__restrict__ nbr_out, uint32_t stride, uint32_t *__restrict__ count,
    uint32_t *__restrict__ retry, uint32_t *nretry)
{
    uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= ntodo) return;
    uint32_t i = todo[t];
    float3 q = make_float3(p[3 * i], p[3 * i + 1], p[3 * i + 2]);
    int3 c = cell_of(g, q);
    Cell C;
    init_box(C, box);
    bool ok = true;
    uint32_t scanned = 0;
    const int rmax = max(g.dim.x, max(g.dim.y, g.dim.z));
    for (int r = 0; r <= rmax && ok; ++r) {
        if (r >= 1) {
            float lim = (float)(r - 1) / g.inv_h;
            if (lim * lim > 4.0f * max_vertex_r2(C)) break;
            if (scanned >= kStreamCap) break;
        }
        for (int z = c.z - r; z <= c.z + r && ok; ++z) {
            if (z < 0 || z >= g.dim.z) continue;
            for (int y = c.y - r; y <= c.y + r && ok; ++y) {
                if (y < 0 || y >= g.dim.y) continue;
                for (int x = c.x - r; x <= c.x + r && ok; ++x) {
                    if (x < 0 || x >= g.dim.x) continue;
                    if (max(abs(x - c.x), max(abs(y - c.y), abs(z - c.z))) != r) continue;
                    uint32_t id = ((uint32_t)z * g.dim.y + y) * g.dim.x + x;
                    for (uint32_t s2 = start[id]; s2 < start[id + 1] && ok; ++s2) {
                        uint32_t j = sorted[s2];
                        if (j == i) continue;
                        float nx = p[3 * j] - q.x, ny = p[3 * j + 1] - q.y, nz = p[3 * j + 2] - q.z;
                        ok = clip(C, make_float4(nx, ny, nz, 0.5f * (nx * nx + ny * ny + nz * nz)), j);
                        ++scanned;
                    }
                }
            }
        }
    }
    if (!ok) {
        uint32_t r = atomicAdd(nretry, 1u);
        retry[r] = i;
        count[i] = 0;
        return;
    }
    count[i] = emit(C, nbr_out + (size_t)i * stride, stride);
}

__global__ void write_csr(const uint32_t *__restrict__ nbr, uint32_t stride,
                          const uint32_t *__restrict__ offs, uint32_t n, uint32_t *__restrict__ adj)
{
    uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint32_t b = offs[i], e = offs[i + 1];
    for (uint32_t k = 0; k < e - b; ++k) adj[b + k] = nbr[(size_t)i * stride + k];
}

inline size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

struct VorWs {
    float *bbox;
    void *mm_scratch;
    uint32_t *cnt, *start, *cell_id, *sorted, *count, *retry, *nretry, *nbr;
    void *temp;
    size_t temp_bytes;
    void *bvh;       // the sites' BVH (vt_bvh_build blob)
    void *bvh_ws;    // its build workspace
};

inline uint32_t grid_cells_bound(uint32_t n) { return 2 * n + 64; }

inline size_t scan_bytes(uint32_t n)
{
    size_t a = 0, b = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, a, (const uint32_t *)nullptr, (uint32_t *)nullptr,
                                  (int)(grid_cells_bound(n) + 1));
    cub::DeviceScan::ExclusiveSum(nullptr, b, (const uint32_t *)nullptr, (uint32_t *)nullptr,
                                  (int)(n + 1));
    return a > b ? a : b;
}

inline VorWs carve(void *ws, uint32_t n)
{
    const uint32_t G = grid_cells_bound(n);
    char *w = (char *)ws;
    VorWs v;
    v.bbox = (float *)w;
    v.mm_scratch = w + 256;
    w += 512;
    v.cnt = (uint32_t *)w;      w += a256((size_t)(G + 1) * 4);
    v.start = (uint32_t *)w;    w += a256((size_t)(G + 1) * 4);
    v.cell_id = (uint32_t *)w;  w += a256((size_t)n * 4);
    v.sorted = (uint32_t *)w;   w += a256((size_t)n * 4);
    v.count = (uint32_t *)w;    w += a256((size_t)(n + 1) * 4);
    v.retry = (uint32_t *)w;    w += 2 * a256((size_t)n * 4);
    v.nretry = (uint32_t *)w;   w += 256;
    v.nbr = (uint32_t *)w;      w += a256((size_t)n * kMaxPlanes * 4);
    v.temp = w;
    v.temp_bytes = scan_bytes(n);
    w += a256(v.temp_bytes);
    v.bvh = w;                  w += a256(vt_bvh_nodes_bytes(n));
    v.bvh_ws = w;
    return v;
}

}  // namespace vor
}  // namespace vt

using namespace vt::vor;

extern "C" uint64_t vt_voronoi_bytes(uint32_t num_points)
{
    const uint32_t n = num_points, G = grid_cells_bound(n);
    return 512 + 2 * a256((size_t)(G + 1) * 4) + 2 * a256((size_t)n * 4) +
           a256((size_t)(n + 1) * 4) + 2 * a256((size_t)n * 4) + 256 +
           a256((size_t)n * kMaxPlanes * 4) + a256(scan_bytes(n)) + a256(vt_bvh_nodes_bytes(n)) +
           vt_bvh_workspace_bytes(n);
}

extern "C" vt_status vt_voronoi_adjacency(const float *points, uint32_t num_points,
                                          const uint32_t *seed_adjacency,
                                          const uint32_t *seed_offsets, void *workspace,
                                          uint64_t workspace_bytes, uint32_t *offsets,
                                          uint64_t *num_entries, uint32_t *unconverged,
                                          vt_stream stream)
{
    const uint32_t n = num_points;
    VT_REQUIRE(points && workspace && offsets && num_entries, "vt_voronoi_adjacency: null pointer");
    VT_REQUIRE(n >= 2, "vt_voronoi_adjacency: need at least 2 sites");
    VT_REQUIRE(!seed_adjacency == !seed_offsets,
               "vt_voronoi_adjacency: seed adjacency and offsets go together");
    VT_REQUIRE(workspace_bytes >= vt_voronoi_bytes(n) && ((uintptr_t)workspace & 255u) == 0,
               "vt_voronoi_adjacency: workspace must be vt_voronoi_bytes large, 256-byte aligned");
    cudaStream_t s = (cudaStream_t)stream;
    VorWs v = carve(workspace, n);
    vt_status st = vt_minmax_f32(points, n, 3, v.mm_scratch, v.bbox, stream);
    if (st != VT_OK) return st;
    float bb[6];
    cudaMemcpyAsync(bb, v.bbox, sizeof(bb), cudaMemcpyDeviceToHost, s);
    cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess)
        return vt::set_error(VT_ERR_CUDA, "vt_voronoi_adjacency: %s", cudaGetErrorString(e));
    float ext[3] = {bb[1] - bb[0], bb[3] - bb[2], bb[5] - bb[4]};
    float emax = fmaxf(ext[0], fmaxf(ext[1], ext[2]));
    if (!(emax > 0.0f))
        return vt::set_error(VT_ERR_INVALID, "vt_voronoi_adjacency: all sites coincide");
    // about 2 sites per grid cell
    double vol = 1.0;
    for (int a = 0; a < 3; ++a) vol *= fmax((double)ext[a], emax * 1e-3);
    double h = cbrt(vol * 2.0 / n);
    Grid g;
    uint64_t G;
    for (;;) {
        g.dim.x = (int)(ext[0] / h) + 1;
        g.dim.y = (int)(ext[1] / h) + 1;
        g.dim.z = (int)(ext[2] / h) + 1;
        G = (uint64_t)g.dim.x * g.dim.y * g.dim.z;
        if (G <= grid_cells_bound(n)) break;
        h *= 1.1;
    }
    g.lo = make_float3(bb[0], bb[2], bb[4]);
    g.inv_h = (float)(1.0 / h);
#ifndef VT_VOR_THREAD_CELLS
#define VT_VOR_THREAD_CELLS 0  // 1: the first pass builds one cell per thread
#endif
#ifndef VT_VOR_BOX
#define VT_VOR_BOX 16.0f  // truncation box half-width in scene extents (measured: 4 -> 16 cuts the
                          // rows missing hull faces 5x for 40 % more build time)
#endif
    const float box = VT_VOR_BOX * emax + 1.0f;
    cudaMemsetAsync(v.cnt, 0, (G + 1) * 4, s);
    grid_count<<<vt::grid_for(n, 256), 256, 0, s>>>(points, n, g, v.cnt, v.cell_id);
    size_t tb = v.temp_bytes;
    cub::DeviceScan::ExclusiveSum(v.temp, tb, v.cnt, v.start, (int)(G + 1), s);
    cudaMemcpyAsync(v.cnt, v.start, (G + 1) * 4, cudaMemcpyDeviceToDevice, s);
    grid_scatter<<<vt::grid_for(n, 256), 256, 0, s>>>(n, v.cell_id, v.cnt, v.sorted);
    grid_sort<<<vt::grid_for(G, 256), 256, 0, s>>>((uint32_t)G, v.start, v.sorted);

    st = vt_bvh_build(points, n, v.bvh, vt_bvh_nodes_bytes(n), v.bvh_ws, vt_bvh_workspace_bytes(n),
                      stream);
    if (st != VT_OK) return st;
    uint32_t *bufs[2] = {v.retry, v.retry + a256((size_t)n * 4) / 4};
    const vt::bvh::Node *nodes = (const vt::bvh::Node *)v.bvh;
    const uint32_t *ids = vt::bvh::leaf_ids(v.bvh, n);
    const uint32_t *todo = nullptr;
    uint32_t ntodo = n;
    // pass 0: every cell; pass 1: failures, seeded with more sites; pass 2:
    // remaining failures, sites streamed ring by ring
    for (int pass = 0; pass < 3 && ntodo > 0; ++pass) {
        uint32_t *out = bufs[pass & 1];
        cudaMemsetAsync(v.nretry, 0, 4, s);
        if (pass == 0 && !VT_VOR_THREAD_CELLS) {
            // one warp per cell, persistent warps taking cells from a counter
            uint32_t *next_cell = v.nretry + 4;
            cudaMemsetAsync(next_cell, 0, 4, s);
            int dev = 0, sms = 148, per_sm = 1;
            cudaGetDevice(&dev);
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, cell_warp_kernel, 32 * kWWarps, 0);
            cell_warp_kernel<<<sms * (per_sm > 0 ? per_sm : 1), 32 * kWWarps, 0, s>>>(
                points, n, g, v.start, v.sorted, nodes, ids, box, seed_adjacency, seed_offsets,
                v.nbr, kMaxPlanes, v.count, out, v.nretry, next_cell);
        } else if (pass < 2)
            cell_verify_kernel<<<vt::grid_for(ntodo, 64), 64, 0, s>>>(
                points, n, g, v.start, v.sorted, nodes, ids, box, todo, ntodo,
                pass == 0 ? kSeedK : kSeedKRetry, pass == 0 ? seed_adjacency : nullptr,
                seed_offsets, v.nbr, kMaxPlanes, v.count, out, v.nretry);
        else
            cell_stream_kernel<<<vt::grid_for(ntodo, 64), 64, 0, s>>>(
                points, n, g, v.start, v.sorted, box, todo, ntodo, v.nbr, kMaxPlanes, v.count,
                out, v.nretry);
        e = cudaGetLastError();
        if (e != cudaSuccess)
            return vt::set_error(VT_ERR_CUDA, "voronoi cell kernel: %s", cudaGetErrorString(e));
        uint32_t nr = 0;
        cudaMemcpyAsync(&nr, v.nretry, 4, cudaMemcpyDeviceToHost, s);
        e = cudaStreamSynchronize(s);
        if (e != cudaSuccess)
            return vt::set_error(VT_ERR_CUDA, "voronoi cell kernel: %s", cudaGetErrorString(e));
#ifdef VT_VOR_VERBOSE
        fprintf(stderr, "voronoi pass %d: %u cells in, %u left\n", pass, ntodo, nr);
#endif
        todo = out;
        ntodo = nr;
    }
    if (unconverged) *unconverged = ntodo;  // cells left empty (degenerate clipping)
    cudaMemsetAsync(v.count + n, 0, 4, s);
    tb = v.temp_bytes;
    cub::DeviceScan::ExclusiveSum(v.temp, tb, v.count, offsets, (int)(n + 1), s);
    uint32_t E = 0;
    cudaMemcpyAsync(&E, offsets + n, 4, cudaMemcpyDeviceToHost, s);
    e = cudaStreamSynchronize(s);
    if (e != cudaSuccess)
        return vt::set_error(VT_ERR_CUDA, "vt_voronoi_adjacency: %s", cudaGetErrorString(e));
    *num_entries = E;
    return VT_OK;
}

extern "C" vt_status vt_voronoi_write(const void *workspace, uint32_t num_points,
                                      const uint32_t *offsets, uint32_t *adjacency, vt_stream stream)
{
    VT_REQUIRE(workspace && offsets && adjacency, "vt_voronoi_write: null pointer");
    VorWs v = carve((void *)workspace, num_points);
    write_csr<<<vt::grid_for(num_points, 256), 256, 0, (cudaStream_t)stream>>>(
        v.nbr, kMaxPlanes, offsets, num_points, adjacency);
    return vt::check_launch("vt_voronoi_write");
}
