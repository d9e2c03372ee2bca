// vt_walk.cuh -- the cell-to-cell walk (reference: tracing_octmap.cu:39-123).
//
// Semantics are the reference's exactly: count the step, stop past
// max_steps, pick the first face in CSR order with dp > 0 and the strictly
// smallest bisector-plane distance t, stop when there is none, integrate the
// segment [t0, t1] only when t1 > t0, and carry t0 = max(t0, t1).
//
// What differs is the schedule.  The reference walk has three dependent
// global loads per cell (CSR offsets -> face offsets -> neighbour id ->
// next offsets).  Here the packed 16-byte face record of the winning face
// carries the neighbour id, its CSR begin and its degree, so the moment a
// cell's exit face is known the walk issues the next cell's first face chunk,
// its site and its density, and only then integrates the current segment
// (texture loads included).  One dependent memory round trip per cell
// remains, and the texture fetch overlaps it.  Face rows are read in chunks
// of kChunk 128-bit loads, two chunk buffers used in turn (the next chunk is
// loaded while the current one is tested, with no register copies), and the
// scan keeps only the winning distance and face index; the winning record is
// read again (an L1 hit) once the row is done.  Measured on the C2 view:
// index tracking + alternating buffers 6.47 -> 5.47 ms, kChunk 4 -> 2 5.36 ms.
#pragma once

#include "vt_geom.cuh"

namespace vt {

struct WalkDebug {
    uint32_t *seq;      // (rays, seq_cap) visited cells, or null
    uint32_t seq_cap;
    uint32_t *seq_len;  // (rays) cells visited (may exceed seq_cap)
    uint4 *stats;       // (rays) steps, faces tested, integrate calls, textured cells
    uint8_t *visited;   // (cells) 1 if any ray visits the cell
    uint8_t *textured;  // (cells) 1 if any ray reads the cell's texels
};

#ifndef VT_CHUNK
#define VT_CHUNK 2
#endif
constexpr uint32_t kChunk = VT_CHUNK;

struct FaceChunk {
    uint4 f[kChunk];
};

__device__ __forceinline__ void load_chunk(FaceChunk &c, const uint4 *__restrict__ row, uint32_t j,
                                           uint32_t deg)
{
#pragma unroll
    for (int k = 0; k < (int)kChunk; ++k)
        if (j + k < deg) c.f[k] = __ldg(row + j + k);
}

struct ExitFace {
    float t1;
    uint32_t nb, nbeg, ndeg;
    bool found;
};

// Winner tracked by index only; the record is re-read (L1) after the row.
__device__ __forceinline__ void test_chunk_idx(const FaceChunk &c, uint32_t j, uint32_t deg, V3 P,
                                               const Ray &ray, float &t1, uint32_t &jbest)
{
#pragma unroll
    for (int k = 0; k < (int)kChunk; ++k) {
        const uint4 f = c.f[k];
        V3 off = mk(h2f((uint16_t)(f.x & 0xffffu)), h2f((uint16_t)(f.x >> 16)),
                    h2f((uint16_t)(f.y & 0xffffu)));
        V3 fo = fma3(off, 0.5f, P);
        float dp = dot(off, ray.d);
        float t = dot(fo - ray.o, off) / dp;
        if (j + k < deg && dp > 0.0f && t < t1) {
            t1 = t;
            jbest = j + k;
        }
    }
}

// Path record of the training forward, replayed by the backward.  Slot k of
// ray r holds the cell entered at walk step k (the exit neighbour found at
// step k) and the colour the forward computed for the segment integrated at
// step k (sigmoid of the sampled logits; 0 when the cell is untextured or the
// segment is empty): {cell, r, g, b bits} in 16 bytes, laid out slot-major
// (steps[k * stride + r]) so that the lanes of a warp, which advance one cell
// per loop iteration together, touch consecutive records.  len[r] = number
// of exit faces found (steps past cap are not stored).
struct PathRec {
    uint4 *steps;
    uint32_t cap;
    uint64_t stride;
    uint32_t *len;
};

// Exit distance through the bisector face shared with site Q.  The packed
// face row of that face holds off = binary16(Q - P) (pack_faces_kernel), so
// this is test_chunk_idx's arithmetic on the same operands, bit for bit.
__device__ __forceinline__ float face_exit_t(V3 P, V3 Q, const Ray &ray)
{
    const V3 d = Q - P;
    const V3 off = mk(h2f(f2h(d.x)), h2f(f2h(d.y)), h2f(f2h(d.z)));
    const V3 fo = fma3(off, 0.5f, P);
    return dot(fo - ray.o, off) / dot(off, ray.d);
}

// Walk state: the cell being entered and everything the next step needs.
struct WalkState {
    uint32_t cur, begin, deg, n;
    V3 P;
    float s, t0;
};

// Integ must provide: bool integrate(uint32_t cell, float t0, float t1,
//                                    V3 P, V3 Q, float density) and
//                     uint32_t textured() const.
// Runs the walk from state w; returns the step count n.
template <class Integ, bool kDebug, bool kRecord>
__device__ __forceinline__ uint32_t walk_from(WalkState w, const Ray &ray,
                                              const uint4 *__restrict__ faces,
                                              const float *__restrict__ points,
                                              const float *__restrict__ density,
                                              uint32_t max_steps, Integ &I, uint32_t ray_id,
                                              const WalkDebug &dbg, const PathRec &rec)
{
    uint32_t cur = w.cur, begin = w.begin, deg = w.deg, n = w.n;
    V3 P = w.P;
    float s = w.s, t0 = w.t0;
    FaceChunk c;
    load_chunk(c, faces + begin, 0, deg);

    uint32_t ns = 0, nfaces = 0, nint = 0, nfound = 0;
    for (;;) {
        n++;
        if (n > max_steps) break;
        if (kDebug) {
            if (dbg.seq && ns < dbg.seq_cap) dbg.seq[(size_t)ray_id * dbg.seq_cap + ns] = cur;
            if (dbg.visited) dbg.visited[cur] = 1;
            ns++;
            nfaces += deg;
        }
        ExitFace x;
        x.t1 = __int_as_float(0x7f800000);
        x.found = false;
        x.nb = x.nbeg = x.ndeg = 0;
        const uint4 *row = faces + begin;
        {
            FaceChunk b;
            uint32_t jbest = 0xffffffffu;
            for (uint32_t j = 0; j < deg; j += 2 * kChunk) {
                load_chunk(b, row, j + kChunk, deg);
                test_chunk_idx(c, j, deg, P, ray, x.t1, jbest);
                if (j + kChunk >= deg) break;
                load_chunk(c, row, j + 2 * kChunk, deg);
                test_chunk_idx(b, j + kChunk, deg, P, ray, x.t1, jbest);
            }
            if (jbest != 0xffffffffu) {
                const uint4 f = __ldg(row + jbest);
                x.nb = f.z;
                x.nbeg = f.w;
                x.ndeg = f.y >> 16;
                x.found = true;
            }
        }

        if (!x.found) break;
        // Issue the next cell's loads before integrating this one.
        V3 Q = ld3(points + (size_t)x.nb * 3);
        float sn = __ldg(density + x.nb);
        load_chunk(c, faces + x.nbeg, 0, x.ndeg);
        bool go = true;
        V3 rgb = mk(0.f, 0.f, 0.f);
        if (x.t1 > t0) {
            if (kDebug) nint++;
            const uint32_t tex_before = kDebug ? I.textured() : 0;
            go = I.integrate(cur, t0, x.t1, P, Q, s);
            if constexpr (kRecord) rgb = I.last_rgb;
            if (kDebug && dbg.textured && I.textured() != tex_before) dbg.textured[cur] = 1;
        }
        if (kRecord) {
            if (nfound < rec.cap)
                rec.steps[(uint64_t)nfound * rec.stride + ray_id] =
                    make_uint4(x.nb, __float_as_uint(rgb.x), __float_as_uint(rgb.y),
                               __float_as_uint(rgb.z));
            nfound++;
        }
        if (!go) break;
        t0 = fmaxf(t0, x.t1);
        cur = x.nb;
        P = Q;
        s = sn;
        begin = x.nbeg;
        deg = x.ndeg;
    }
    if (kDebug) {
        if (dbg.seq_len) dbg.seq_len[ray_id] = ns;
        if (dbg.stats) dbg.stats[ray_id] = make_uint4(ns, nfaces, nint, I.textured());
    }
    if (kRecord && rec.len) rec.len[ray_id] = nfound;
    return n;
}

template <class Integ, bool kDebug, bool kRecord = false>
__device__ __forceinline__ uint32_t walk(const Ray &ray, const uint4 *__restrict__ faces,
                                         const uint32_t *__restrict__ offs,
                                         const float *__restrict__ points,
                                         const float *__restrict__ density, uint32_t start,
                                         uint32_t max_steps, Integ &I, uint32_t ray_id,
                                         const WalkDebug &dbg,
                                         const PathRec &rec = PathRec{nullptr, 0, 0, nullptr})
{
    WalkState w;
    w.cur = start;
    w.begin = __ldg(offs + start);
    w.deg = __ldg(offs + start + 1) - w.begin;
    w.P = ld3(points + (size_t)start * 3);
    w.s = __ldg(density + start);
    w.t0 = 0.0f;
    w.n = 0;
    return walk_from<Integ, kDebug, kRecord>(w, ray, faces, points, density, max_steps, I, ray_id,
                                             dbg, rec);
}

// Flag in PathRec::len: the backward must walk this ray itself (the record
// overflowed, or the forward stopped at T == weight_threshold exactly, where
// the backward's stop rule T < weight_threshold lets the walk go on).
constexpr uint32_t kPathWalk = 0x80000000u;

// Backward replay: the cells of the forward's path record are entered
// without scanning faces (the exit distance is recomputed from the two
// sites), and each segment's colour is the forward's, so no texel is read
// back (Integ::integrate_recorded).  The walk is deterministic, so every recorded step is the step the
// scan would take, and an unflagged record ends where the backward's walk
// ends (no exit face, the step limit, or T < weight_threshold, which stopped
// the forward at the same step).  Returns false if the integrator stopped the
// walk, else true with w set to the walk state after the recorded steps
// (begin / deg left for the caller), from which a flagged ray's walk goes on.
// The record of step k+2 and the site of step k+1 are loaded one iteration
// ahead.
template <class Integ>
__device__ __forceinline__ bool walk_replay(const Ray &ray, const float *__restrict__ points,
                                            const float *__restrict__ density, uint32_t start,
                                            uint32_t L, Integ &I, const uint4 *steps,
                                            uint64_t stride, WalkState &w)
{
    uint32_t cur = start;
    V3 P = ld3(points + (size_t)start * 3);
    float s = __ldg(density + start);
    float t0 = 0.0f;
    uint4 st = make_uint4(0, 0, 0, 0), st1 = make_uint4(0, 0, 0, 0);
    V3 Q = P;
    float sq = 0.0f;
    if (L > 0) {
        st = __ldg(steps);
        Q = ld3(points + (size_t)st.x * 3);
        sq = __ldg(density + st.x);
    }
    if (L > 1) st1 = __ldg(steps + stride);
    for (uint32_t k = 0; k < L; ++k) {
        V3 Qn = Q;
        float sqn = 0.0f;
        uint4 st2 = make_uint4(0, 0, 0, 0);
        if (k + 1 < L) {
            Qn = ld3(points + (size_t)st1.x * 3);
            sqn = __ldg(density + st1.x);
        }
        if (k + 2 < L) st2 = __ldg(steps + (uint64_t)(k + 2) * stride);
        const float t1 = face_exit_t(P, Q, ray);
        if (t1 > t0) {
            const V3 rgb = mk(__uint_as_float(st.y), __uint_as_float(st.z), __uint_as_float(st.w));
            if (!I.integrate_recorded(cur, t0, t1, P, Q, s, rgb)) return false;
        }
        t0 = fmaxf(t0, t1);
        cur = st.x;
        P = Q;
        s = sq;
        st = st1;
        Q = Qn;
        sq = sqn;
        st1 = st2;
    }
    w.cur = cur;
    w.P = P;
    w.s = s;
    w.t0 = t0;
    w.n = L;
    return true;
}

}  // namespace vt
