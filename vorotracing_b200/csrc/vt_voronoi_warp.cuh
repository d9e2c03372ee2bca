// vt_voronoi_warp.cuh -- one warp per Voronoi cell, the cell in shared memory.
//
// Included by vt_voronoi.cu (it uses that file's Grid, cell_of, solve3 and
// the sites' BVH).  Same method as cell_verify_kernel: clip a box by the
// bisector planes of nearby sites, then verify every vertex by the
// empty-ball property through the BVH, clipping by any site found inside a
// vertex's ball.  The difference is the execution: a thread per cell keeps
// its cell (about 9 KB) in local memory, and the lanes of a warp, each on its
// own cell, diverge on every loop (3.5 of 32 lanes active, 92 GB of local
// memory traffic for 1M cells).  Here the 32 lanes build one cell together:
//   * a clip tests the vertices 32 at a time (ballots give the removed set),
//     collects the boundary edges with a warp-aggregated append, finds free
//     vertex slots with one bit search per lane, and closes the hole with one
//     lane per new vertex (each solving its 3x3 system);
//   * verification runs one BVH ball search per lane (32 vertices at a
//     time), then clips by the sites found, one after the other;
//   * seeding scans the grid cells of the first rings, one cell per lane,
//     and orders the candidates by a parallel rank.
// The vertex / plane bookkeeping is the dual triangle structure of Cell,
// with the live and verified sets as bit masks.
#pragma once

namespace vt {
namespace vor {

#ifndef VT_VOR_WTRIS
#define VT_VOR_WTRIS 127  // measured: 255 -> 127 slots (and 128 -> 64 planes) 0.134 -> 0.117 s for 1M sites: more warps per SM
#endif
#ifndef VT_VOR_WPLANES
#define VT_VOR_WPLANES 64
#endif
constexpr int kWTris = VT_VOR_WTRIS;  // vertex slots (uint8 ids, 255 = none)
constexpr int kWWords = (kWTris + 1) / 32;  // 32-bit mask words covering the slots
constexpr int kWPlanes = VT_VOR_WPLANES;
constexpr int kWRing = 128;      // boundary edges of one clip
constexpr int kWCand = 128;      // seed candidates
#ifndef VT_VOR_WSEEDS
#define VT_VOR_WSEEDS 32  // measured: 12, 16, 24, 32 -> 0.147, 0.146, 0.141, 0.135 s for 1M sites
#endif
constexpr int kWSeeds = VT_VOR_WSEEDS;
constexpr int kWWarps = 4;       // warps per block
constexpr int kWMaxClips = 768;
constexpr int kWMaxRounds = 2048;
constexpr unsigned kFull = 0xffffffffu;

struct WCell {
    float4 plane[kWPlanes];      // n.xyz, d: n.x <= d inside
    uint32_t site[kWPlanes];     // neighbour id, 0xffffffff for the box
    float4 pos[kWTris + 1];      // vertex positions (relative to the site)
    uchar4 tri[kWTris + 1];      // plane ids (x, y, z), counter-clockwise from outside
    uchar4 nbr[kWTris + 1];      // vertex across edge (v0v1, v1v2, v2v0)
    uint32_t alive[kWWords];
    uint32_t verified[kWWords];
    uint32_t out[kWWords];
    uint32_t fresh[kWWords];     // slots (re)filled since the verification round began
    uint32_t used[kWPlanes / 32];
    int start_of[kWPlanes];
    uint8_t ea[kWRing], eb[kWRing], en[kWRing], slot_of[kWRing];
    uint32_t cand[kWCand];
    float cand_d[kWCand];
    int ntris, nplanes, ncand;
};

__device__ __forceinline__ uint8_t uc(const uchar4 &v, int k)
{
    return k == 0 ? v.x : (k == 1 ? v.y : v.z);
}
__device__ __forceinline__ void set_uc(uchar4 &v, int k, uint8_t x)
{
    if (k == 0)
        v.x = x;
    else if (k == 1)
        v.y = x;
    else
        v.z = x;
}
__device__ __forceinline__ bool bit(const uint32_t *m, int t) { return (m[t >> 5] >> (t & 31)) & 1u; }
// Position of the k-th (0-based) set bit of m; requires popc(m) > k.
__device__ __forceinline__ int nth_set_bit(unsigned m, int k)
{
    int pos = 0;
    for (int s = 16; s > 0; s >>= 1) {
        const unsigned low = m & ((1u << s) - 1u);
        const int c = __popc(low);
        if (k >= c) {
            k -= c;
            m >>= s;
            pos += s;
        } else {
            m = low;
        }
    }
    return pos;
}
// byte-wise neighbour update: several lanes may update different edges of
// one vertex in the same step
__device__ __forceinline__ void set_nb(WCell &C, int t, int k, uint8_t v)
{
    reinterpret_cast<uint8_t *>(&C.nbr[t])[k] = v;
}

// Box of half-width B around the site: 6 planes, 8 vertices.
__device__ void wc_init_box(WCell &C, float B, int lane)
{
    const float4 P[6] = {{1, 0, 0, B}, {-1, 0, 0, B}, {0, 1, 0, B},
                         {0, -1, 0, B}, {0, 0, 1, B}, {0, 0, -1, B}};
    const uchar4 T[8] = {{0, 2, 4, 0}, {0, 5, 2, 0}, {0, 3, 5, 0}, {0, 4, 3, 0},
                         {1, 4, 2, 0}, {1, 2, 5, 0}, {1, 5, 3, 0}, {1, 3, 4, 0}};
    const uchar4 N[8] = {{1, 4, 3, 0}, {2, 5, 0, 0}, {3, 6, 1, 0}, {0, 7, 2, 0},
                         {7, 0, 5, 0}, {4, 1, 6, 0}, {5, 2, 7, 0}, {6, 3, 4, 0}};
    if (lane < 6) {
        C.plane[lane] = P[lane];
        C.site[lane] = 0xffffffffu;
    }
    if (lane < 8) {
        float3 x;
        solve3(P[T[lane].x], P[T[lane].y], P[T[lane].z], x);
        C.pos[lane] = make_float4(x.x, x.y, x.z, 0.0f);
        C.tri[lane] = T[lane];
        C.nbr[lane] = N[lane];
    }
    if (lane < kWWords) {
        C.alive[lane] = lane == 0 ? 0xffu : 0u;
        C.verified[lane] = 0u;
        C.out[lane] = 0u;
        C.fresh[lane] = 0u;
    }
    if (lane == 0) {
        C.ntris = 8;
        C.nplanes = 6;
    }
    __syncwarp();
}

// Drop planes no live vertex uses (box planes stay at 0..5).  Lane-parallel
// marking, lane-0 renumbering (rare: only when the plane table is full).
__device__ void wc_compact_planes(WCell &C, int lane)
{
    if (lane < kWPlanes / 32) C.used[lane] = lane == 0 ? 0x3fu : 0u;
    __syncwarp();
    for (int t = lane; t < C.ntris; t += 32)
        if (bit(C.alive, t)) {
            const uchar4 v = C.tri[t];
            atomicOr(&C.used[v.x >> 5], 1u << (v.x & 31));
            atomicOr(&C.used[v.y >> 5], 1u << (v.y & 31));
            atomicOr(&C.used[v.z >> 5], 1u << (v.z & 31));
        }
    __syncwarp();
    if (lane == 0) {
        uint8_t remap[kWPlanes];
        int k = 0;
        for (int p = 0; p < C.nplanes; ++p) {
            remap[p] = (uint8_t)k;
            if (bit(C.used, p)) {
                C.plane[k] = C.plane[p];
                C.site[k] = C.site[p];
                ++k;
            }
        }
        for (int t = 0; t < C.ntris; ++t)
            if (bit(C.alive, t)) {
                uchar4 v = C.tri[t];
                v.x = remap[v.x];
                v.y = remap[v.y];
                v.z = remap[v.z];
                C.tri[t] = v;
            }
        C.nplanes = k;
    }
    __syncwarp();
}

// Clip the cell by plane pl of site j (whole warp).  Returns 1 if vertices
// were removed, 0 if the plane misses the cell, -1 if clipping failed
// (overflow or a degenerate configuration).
__device__ int wc_clip(WCell &C, float4 pl, uint32_t j, int lane)
{
    const unsigned lt = (1u << lane) - 1u;
    const int nt = C.ntris;
    const int nw = (nt + 31) >> 5;
    int nout = 0, nin = 0;
    for (int w = 0; w < nw; ++w) {
        const int t = w * 32 + lane;
        const bool al = t < nt && ((C.alive[w] >> lane) & 1u);
        bool o = false;
        if (al) {
            const float4 p = C.pos[t];
            o = pl.x * p.x + pl.y * p.y + pl.z * p.z - pl.w > 0.0f;
        }
        const unsigned om = __ballot_sync(kFull, o);
        const unsigned am = __ballot_sync(kFull, al);
        if (lane == 0) C.out[w] = om;
        nout += __popc(om);
        nin += __popc(am & ~om);
    }
    __syncwarp();
    if (nout == 0) return 0;
    if (nin == 0) return -1;
    if (C.nplanes >= kWPlanes) {
        wc_compact_planes(C, lane);
        if (C.nplanes >= kWPlanes) return -1;
    }
    const int np = C.nplanes;
    // boundary edges a -> b of removed vertices whose neighbour survives
    bool bad = false;
    int ne = 0;
    for (int w = 0; w < nw; ++w) {
        const int t = w * 32 + lane;
        const bool o = (C.out[w] >> lane) & 1u;
        uchar4 tv = make_uchar4(0, 0, 0, 0), nv = tv;
        if (o) {
            tv = C.tri[t];
            nv = C.nbr[t];
        }
        for (int k = 0; k < 3; ++k) {
            bool isb = false;
            if (o) {
                const uint8_t n = uc(nv, k);
                if (n == 0xff)
                    bad = true;
                else if (!bit(C.out, n))
                    isb = true;
            }
            const unsigned bm = __ballot_sync(kFull, isb);
            const int pos = ne + __popc(bm & lt);
            if (isb && pos < kWRing) {
                C.ea[pos] = uc(tv, k);
                C.eb[pos] = uc(tv, (k + 1) % 3);
                C.en[pos] = uc(nv, k);
            }
            ne += __popc(bm);
        }
    }
    if (__any_sync(kFull, bad) || ne > kWRing || ne < 3) return -1;
    // remove the cut vertices, free slots for the new ones
    if (lane < nw) C.alive[lane] &= ~C.out[lane];
    for (int p = lane; p <= np; p += 32) C.start_of[p] = -1;
    if (lane == 0) {
        C.plane[np] = pl;
        C.site[np] = j;
    }
    __syncwarp();
    int nfree = 0;
    for (int w = 0; w < nw; ++w) {
        const unsigned valid = (w == (nt >> 5)) ? ((1u << (nt & 31)) - 1u) : kFull;
        nfree += __popc(~C.alive[w] & valid);
    }
    const int new_nt = nt + (ne > nfree ? ne - nfree : 0);
    if (new_nt > kWTris) return -1;
    // slot of edge e: the e-th free slot below nt, else appended (all slots
    // are chosen before any is taken)
    for (int e = lane; e < ne; e += 32) {
        int slot = -1, acc = 0;
        for (int w = 0; w < nw && slot < 0; ++w) {
            const unsigned valid = (w == (nt >> 5)) ? ((1u << (nt & 31)) - 1u) : kFull;
            const unsigned f = ~C.alive[w] & valid;
            const int c = __popc(f);
            if (e < acc + c) slot = w * 32 + nth_set_bit(f, e - acc);
            acc += c;
        }
        if (slot < 0) slot = nt + (e - nfree);
        C.slot_of[e] = (uint8_t)slot;
    }
    __syncwarp();
    for (int e = lane; e < ne; e += 32) {
        const int slot = C.slot_of[e];
        const uint8_t a = C.ea[e], b = C.eb[e], n = C.en[e];
        float3 x;
        if (!solve3(C.plane[a], C.plane[b], pl, x)) bad = true;
        C.tri[slot] = make_uchar4(a, b, (uint8_t)np, 0);
        C.nbr[slot] = make_uchar4(n, 0xff, 0xff, 0);
        C.pos[slot] = make_float4(x.x, x.y, x.z, 0.0f);
        const uchar4 tn = C.tri[n];
        for (int m = 0; m < 3; ++m)
            if (uc(tn, m) == b && uc(tn, (m + 1) % 3) == a) set_nb(C, n, m, (uint8_t)slot);
        if (atomicExch(&C.start_of[a], e) != -1) bad = true;  // boundary not a simple cycle
        atomicOr(&C.alive[slot >> 5], 1u << (slot & 31));
        atomicAnd(&C.verified[slot >> 5], ~(1u << (slot & 31)));
        atomicOr(&C.fresh[slot >> 5], 1u << (slot & 31));
    }
    __syncwarp();
    // fan around the new plane: (a, b, np) is followed by the vertex whose
    // boundary edge starts at b
    for (int e = lane; e < ne; e += 32) {
        const int f = C.start_of[C.eb[e]];
        if (f < 0) {
            bad = true;
        } else {
            set_nb(C, C.slot_of[e], 1, C.slot_of[f]);
            set_nb(C, C.slot_of[f], 2, C.slot_of[e]);
        }
    }
    if (lane == 0) {
        C.ntris = new_nt;
        C.nplanes = np + 1;
    }
    __syncwarp();
    return __any_sync(kFull, bad) ? -1 : 1;
}

// A site (other than i and the skipped ones) closer to vertex v than site
// i, by the clip's own plane test, or 0xffffffff.  BVH traversal as in
// bvh_cut, without clipping.
__device__ uint32_t bvh_find(const float *__restrict__ p, uint32_t i, float3 q, float3 v,
                             const bvh::Node *__restrict__ nodes, const uint32_t *__restrict__ ids,
                             uint32_t skip0, uint32_t skip1, uint32_t skip2, bool &overflow)
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
                const float w = 0.5f * (nx * nx + ny * ny + nz * nz);
                if (nx * v.x + ny * v.y + nz * v.z - w > 0.0f) return j;
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
                if (sp >= bvh::kStack) {
                    overflow = true;
                    return 0xffffffffu;
                }
                stack[sp++] = c[1 - nearf];
            }
            if (dd[nearf] <= lim) {
                cur = c[nearf];
                continue;
            }
        }
        if (sp == 0) return 0xffffffffu;
        cur = stack[--sp];
    }
}

__device__ __forceinline__ float4 bisector(const float *__restrict__ p, float3 q, uint32_t j)
{
    const float nx = p[3 * j] - q.x, ny = p[3 * j + 1] - q.y, nz = p[3 * j + 2] - q.z;
    return make_float4(nx, ny, nz, 0.5f * (nx * nx + ny * ny + nz * nz));
}

// One warp per cell, cells taken from a global counter.  Cells that fail go
// to the retry list (the thread-per-cell kernels rebuild them).
__global__ void __launch_bounds__(32 * kWWarps) cell_warp_kernel(
    const float *__restrict__ p, uint32_t n, Grid g, const uint32_t *__restrict__ start,
    const uint32_t *__restrict__ sorted, const bvh::Node *__restrict__ nodes,
    const uint32_t *__restrict__ ids, float box, const uint32_t *__restrict__ seed_adj,
    const uint32_t *__restrict__ seed_offs, uint32_t *__restrict__ nbr_out, uint32_t stride,
    uint32_t *__restrict__ count, uint32_t *__restrict__ retry, uint32_t *nretry,
    uint32_t *next_cell)
{
    __shared__ WCell cells[kWWarps];
    const int lane = threadIdx.x & 31;
    WCell &C = cells[threadIdx.x >> 5];
    for (;;) {
        uint32_t i = 0;
        if (lane == 0) i = atomicAdd(next_cell, 1u);
        i = __shfl_sync(kFull, i, 0);
        if (i >= n) return;
        const float3 q = make_float3(p[3 * i], p[3 * i + 1], p[3 * i + 2]);
        wc_init_box(C, box, lane);
        // seed candidates: the caller's guesses, else the sites of the grid
        // rings around the site until kWSeeds are found
        if (lane == 0) C.ncand = 0;
        __syncwarp();
        if (seed_adj) {
            const uint32_t b = seed_offs[i], e = seed_offs[i + 1];
            for (uint32_t k = b + lane; k < e; k += 32) {
                const uint32_t j = seed_adj[k];
                if (j >= n || j == i) continue;
                const int pos = atomicAdd(&C.ncand, 1);
                if (pos < kWCand) {
                    const float4 pl = bisector(p, q, j);
                    C.cand[pos] = j;
                    C.cand_d[pos] = 2.0f * pl.w;
                }
            }
            __syncwarp();
        } else {
            const int3 c = cell_of(g, q);
            for (int r = 0; r <= 3; ++r) {
                const int side = 2 * r + 1, cube = side * side * side;
                for (int idx = lane; idx < cube; idx += 32) {
                    const int dx = idx % side - r, dy = (idx / side) % side - r, dz = idx / (side * side) - r;
                    if (max(abs(dx), max(abs(dy), abs(dz))) != r) continue;
                    const int x = c.x + dx, y = c.y + dy, z = c.z + dz;
                    if (x < 0 || y < 0 || z < 0 || x >= g.dim.x || y >= g.dim.y || z >= g.dim.z)
                        continue;
                    const uint32_t id = ((uint32_t)z * g.dim.y + y) * g.dim.x + x;
                    for (uint32_t s = start[id]; s < start[id + 1]; ++s) {
                        const uint32_t j = sorted[s];
                        if (j == i) continue;
                        const int pos = atomicAdd(&C.ncand, 1);
                        if (pos >= kWCand) break;
                        const float4 pl = bisector(p, q, j);
                        C.cand[pos] = j;
                        C.cand_d[pos] = 2.0f * pl.w;
                    }
                }
                __syncwarp();
                if (C.ncand >= kWSeeds && r >= 1) break;
            }
        }
        const int m = min(C.ncand, kWCand);
        // rank the candidates by (distance, id); clip by the nearest kWSeeds in order
        uint32_t my_j[kWCand / 32];
        int my_rank[kWCand / 32];
        for (int k = 0; k < kWCand / 32; ++k) {
            const int a = k * 32 + lane;
            my_rank[k] = kWCand;
            my_j[k] = 0;
            if (a < m) {
                const float da = C.cand_d[a];
                const uint32_t ja = C.cand[a];
                int r = 0;
                for (int b = 0; b < m; ++b) {
                    const float db = C.cand_d[b];
                    r += (db < da || (db == da && C.cand[b] < ja)) ? 1 : 0;
                }
                my_rank[k] = r;
                my_j[k] = ja;
            }
        }
        __syncwarp();
        for (int k = 0; k < kWCand / 32; ++k)
            if (my_rank[k] < kWSeeds) C.cand[my_rank[k]] = my_j[k];
        __syncwarp();
        bool ok = true;
        int clips = 0;
        const int nseed = min(m, kWSeeds);
        for (int s = 0; s < nseed && ok; ++s) {
            const uint32_t j = C.cand[s];
            ok = wc_clip(C, bisector(p, q, j), j, lane) >= 0;
        }
        // verification rounds: one vertex per lane (bounded: a cell that
        // needs more goes to the retry list)
        for (int round = 0; ok; ++round) {
            if (round >= kWMaxRounds) {
                ok = false;
                break;
            }
            if (lane < kWWords) C.fresh[lane] = 0u;
            __syncwarp();
            int t = -1;
            for (int w = 0; w < (C.ntris + 31) >> 5 && t < 0; ++w) {
                const unsigned todo = C.alive[w] & ~C.verified[w];
                // lane takes the lane-th unverified vertex of the word, if any
                if ((int)__popc(todo) > lane) t = w * 32 + nth_set_bit(todo, lane);
            }
            const bool has = t >= 0 && t < C.ntris;
            if (!__any_sync(kFull, has)) break;
            uint32_t found = 0xffffffffu;
            bool overflow = false;
            if (has) {
                const uchar4 tv = C.tri[t];
                const float4 v = C.pos[t];
                found = bvh_find(p, i, q, make_float3(v.x, v.y, v.z), nodes, ids, C.site[tv.x],
                                 C.site[tv.y], C.site[tv.z], overflow);
            }
            if (__any_sync(kFull, overflow)) {
                ok = false;
                break;
            }
            __syncwarp();
            if (has && found == 0xffffffffu) atomicOr(&C.verified[t >> 5], 1u << (t & 31));
            __syncwarp();
            unsigned fm = __ballot_sync(kFull, found != 0xffffffffu);
            while (fm && ok) {
                const int src = __ffs(fm) - 1;
                fm &= fm - 1;
                const uint32_t j = __shfl_sync(kFull, found, src);
                const int tsrc = __shfl_sync(kFull, t, src);
                // a site whose plane already bounds the cell cuts the vertex
                // only by rounding: the vertex counts as verified
                bool dup = false;
                for (int base = 0; base < C.nplanes; base += 32) {
                    const int pp = base + lane;
                    dup |= pp < C.nplanes && C.site[pp] == j;
                }
                if (__any_sync(kFull, dup)) {
                    // (only if the slot still holds the vertex that found j)
                    if (lane == 0 && bit(C.alive, tsrc) && !bit(C.fresh, tsrc))
                        atomicOr(&C.verified[tsrc >> 5], 1u << (tsrc & 31));
                    __syncwarp();
                    continue;
                }
                // a miss means the vertex that found j is gone already
                ok = wc_clip(C, bisector(p, q, j), j, lane) >= 0;
                if (++clips > kWMaxClips) ok = false;
            }
        }
        if (!ok) {
            if (lane == 0) {
                retry[atomicAdd(nretry, 1u)] = i;
                count[i] = 0;
            }
            __syncwarp();
            continue;
        }
        // emit the neighbour ids of the planes still bounding the cell, ascending
        if (lane < kWPlanes / 32) C.used[lane] = 0u;
        __syncwarp();
        for (int t = lane; t < C.ntris; t += 32)
            if (bit(C.alive, t)) {
                const uchar4 v = C.tri[t];
                atomicOr(&C.used[v.x >> 5], 1u << (v.x & 31));
                atomicOr(&C.used[v.y >> 5], 1u << (v.y & 31));
                atomicOr(&C.used[v.z >> 5], 1u << (v.z & 31));
            }
        __syncwarp();
        int nn = 0;
        for (int base = 6; base < C.nplanes; base += 32) {
            const int pp = base + lane;
            const bool u = pp < C.nplanes && bit(C.used, pp);
            const unsigned um = __ballot_sync(kFull, u);
            if (u) C.cand[nn + __popc(um & ((1u << lane) - 1u))] = C.site[pp];
            nn += __popc(um);
        }
        __syncwarp();
        nn = min(nn, (int)stride);
        uint32_t *out = nbr_out + (size_t)i * stride;
        for (int a = lane; a < nn; a += 32) {
            const uint32_t ja = C.cand[a];
            int r = 0;
            for (int b = 0; b < nn; ++b) r += C.cand[b] < ja ? 1 : 0;
            out[r] = ja;
        }
        if (lane == 0) count[i] = (uint32_t)nn;
        __syncwarp();
    }
}

}  // namespace vor
}  // namespace vt
