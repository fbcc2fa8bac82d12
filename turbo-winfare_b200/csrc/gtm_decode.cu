// Fused batch-1 MoE decode for sm_100a: one persistent cooperative launch runs a token through
// `num_layers` MoE blocks with every expert resident in HBM and no host round trip.
//
// Replaces the per-layer MoE sequence of ForwardRunner::produce_token (src/runner.cpp:549-716):
// MulBF16 -> GemvInt8 -> RouterTopK -> CPU read-back -> shared expert (GemvInt4 x3, GeGLU,
// RMSNormK) -> per expert GemvInt4 gate/up, GeGLU, GemvInt4 down, ScaleAccum -> LayerTail.
//
// Weight streaming. Each CTA (one per SM) has a fixed list of weight "chunks" per layer: its
// router row, its shared gate/up tiles, its routed gate/up tiles (the expert ids come from the
// layer's top-8) and its down rows. A producer warp copies them with cp.async.bulk (the TMA's
// global -> shared bulk copy, one instruction per contiguous range) into a 144 KB shared-memory
// ring, in the order the compute warps use them, as far ahead as the ring has room. So the static
// weights of the next phase or layer stream in while the CTA waits at a grid barrier or works
// through the layer tail, and the routed weights are all requested the moment the top-8 is known.
// The 22 compute warps wait on each chunk's mbarrier and hand it back to the producer with an
// arrival on the chunk's "empty" mbarrier.
//
// Int4 products. A 16-row tile is processed one "quad" of 4 quantisation groups (128 bytes of a
// row) at a time. Lane (g, t) of a warp loads 16 bytes of row g and 16 of row g + 8 per double
// group h (bytes 64 h + 16 t of the quad): rows of 1408 bytes start on the same bank, so gate/up
// tiles put 4 gate rows and 4 up rows in each half of the tile, and the up rows sit 64 bytes off
// the gate rows in shared memory; down rows (352 and 1056 bytes) land on four bank offsets by
// themselves. Every 16-byte load of a warp is then conflict-free. The products are integer
// tensor-core MMAs (mma.sync.m16n8k32, u8 x s8 -> s32): a word of 8 nibbles becomes two registers
// of four u8 (w & 0x0F0F0F0F and (w >> 4) & 0x0F0F0F0F), the A operand of rows g and g + 8. The
// activation enters as the B operand: each group of 64 is written as x = 2^(E-6) (L0 + L1 / 2^7
// + L2 / 2^14) with a power-of-two group scale (|x| < 2^E) and three signed limbs of at most 64
// in magnitude, so each x is carried to 2^-21 of the group's largest; the limbs of the two groups
// of a double group sit in B columns 0-2 and 4-6. Integer accumulation is exact, so D holds per
// row and group the three limb sums of sum_k q_k x_k exactly. After a double group the lane pair
// holding a group combines them in fp32 and applies the group's bf16 scale and bias:
// y += s * 2^(E-6) * (D0 + D1 2^-7 + D2 2^-14) + b * sum(x).
//
// The grid splits into the shared-expert group (40 of 148 CTAs) and eight slot groups (13-14 CTAs
// each, one per top-8 slot). Per layer (one token), with bounded waits:
//   tail    every CTA: layer tail of the previous layer from the down rows, optional
//           between-layer RMSNorm, views (dense_x, routed_x, router input), the group's view table
//   router  CTAs 0..127: their router logit in the reference's exact order (bit-identical), published
//           with the layer number in one 64-bit word; the words double as barrier A
//   slots   wait for all 128 logit words, top-8; the producer starts the slot expert's copies;
//           the group's share of the expert's 88 gate/up tiles (+GeGLU) -> the group's barrier;
//           fragment tables of the expert's 704 activations; the group's share of its 176 down
//           row tiles, each over the whole K                                  -> barrier C
//   shared  the group's share of the 264 shared gate/up tiles (+GeGLU) -> the group's barrier;
//           tables of the 2112 activations; its share of the 176 down row tiles (K 2112); then the
//           top-8 (the tail's weights)                                        -> barrier C
// Every down row comes from one CTA: part [shared, slot 0..7][2816]; the tail weights and sums the
// slots in router order.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "gtm_common.cuh"
#include "gtm_frag.cuh"
#include "gtm_internal.h"
#include "gtm_tcgen05.cuh"

namespace gtm {
namespace dec {

constexpr int D = 2816, FE = 704, FS = 2112, NE = 128, TOPK = 8;
constexpr int NWC = 22;                   // compute warps
constexpr int NTC = NWC * 32;             // 704 compute threads: one float4 of a hidden vector each
constexpr int NT = NTC + 32;              // + the producer warp
constexpr int GD = D / kGroup;            // 44 groups in a hidden-sized input
constexpr int GFE = FE / kGroup;          // 11
constexpr int GFS = FS / kGroup;          // 33
constexpr int QD = GD / 4;                // 11 quads of a hidden-sized input
constexpr int QS = 3;                     // quads of an 11-group down segment (the last holds 3 groups)
constexpr int TILES_S = FS / 8;           // 264 shared gate/up tiles
constexpr int TPE = FE / 8;               // 88 tiles per routed expert
constexpr int OT = D / 16;                // 176 output row tiles of the down projection
constexpr int ROW_GU = D / 2;             // 1408 bytes per gate/up row
constexpr int SROW_GU = GD * 2;           // 88 bytes of bf16 scales per gate/up row
constexpr int DROW_R = FE / 2, SROW_R = GFE * 2;   // routed down: 352 bytes per row, 22 of scales
constexpr int DROW_S = FS / 2, SROW_S = GFS * 2;   // shared down: 1056, 66
constexpr int RIN_PITCH = 65;
constexpr int QW = 192;                   // fragment-table words per quad: 2 double groups x 12 lane entries x 8
constexpr uint32_t RING = 144 * 1024;     // chunk ring
constexpr int NB = 32;                    // chunk mbarrier slots (> the chunks of any one phase)
constexpr int GU_TILES = 1;               // tiles per gate/up chunk
constexpr int DN_TILES_R = 6, DN_TILES_S = 3;   // down row tiles per chunk (38 KB routed, 57 KB shared)
constexpr int MAX_DN = 24;                // items of one phase per CTA (tiles or down row tiles)
constexpr int QSS = 9;                    // quads of the shared down's 33 groups (the last holds 1)
constexpr int MIN_CTAS = 120, MAX_CTAS = 176;   // grid sizes whose per-CTA chunks fit the ring
constexpr int ACT_R = TOPK * FE;          // 5632 routed activations, after the 2112 shared ones
constexpr int SLOTS = 1024;               // partial-sum floats: items x max contributors x 16 rows
constexpr uint64_t kTimeoutNs = 2000000000ull;

struct Params {
    GtmLayer layers[GTM_MAX_LAYERS];
    GtmDecodeIO io;
    int num_layers;
    float eps;
    float inv_sqrt_d;
    unsigned long long* logit_words;   // [NE]: (layer + 1) << 32 | logit bits
    unsigned* flags_b;                 // [256] barrier B, one word per CTA
    unsigned* flags_c;                 // [256] barrier C
    uint64_t wait_limit_ns;            // bound of every wait
    unsigned first_wait_extra;         // added to the first wait's epoch (test hook: 1 = never reached)
    int* err;
    int* sticky;
    float* act;        // [FS + ACT_R]: shared activations, then the 8 routed slots (segment q at q * 704)
    float* part;       // [1 + TOPK][D]: the shared down, then the routed down of slot k (unweighted)
};

// Per-CTA work lists (identical on every thread; derived from the CTA index and grid size). The
// grid splits into the shared-expert group (CTAs [0, S)) and one group per top-8 slot (the rest,
// in eight near-equal ranges): a group computes its expert's gate/up tiles, waits for its own
// members only, then the expert's down rows over the whole K, so every down output row comes from
// one CTA.
struct Plan {
    int nr;              // router rows: cta, cta + G, ...
    bool sh;             // shared-expert group (else the group of top-8 slot `slot`)
    int slot;
    int g0, g1;          // the group's CTAs (its barrier)
    int t0, t1;          // gate/up tiles: of the shared expert's 264, or of the slot expert's 88
    int ot0, ot1;        // down row tiles, each over the expert's whole K (33 or 11 groups)
    int n_gu, n_dn;      // gate/up chunks, down chunks
    int dt;              // down row tiles per down chunk
    int c_gu, c_dn, cpl; // first gate/up chunk, first down chunk, chunks per layer
};
__host__ __device__ constexpr int shared_ctas(int G) { return G * 40 / 148; }

struct Smem {
    alignas(128) uint8_t ring[RING + 128];   // chunks (+ slack read by a down row's partial last quad)
    alignas(16) float hid[D];
    union {
        struct {
            alignas(16) float ab[2 * D];     // routed_x [0, D), dense_x [D, 2D)
            alignas(16) float rin[GD * RIN_PITCH];
        } t;
        alignas(16) uint32_t tbl_dn[QSS * QW];         // down inputs: 33 (shared) or 11 (routed) groups
    } u;
    alignas(16) uint32_t tbl_r[QD * QW];     // routed_x
    alignas(16) uint32_t tbl_d[QD * QW];     // dense_x
    float2 gs_r[GD], gs_d[GD];               // per group of the views: (sum of x, 2^(E-6))
    float2 gs_dn[4 * QSS];                   // and of the down inputs
    float slot[SLOTS];                       // partial sums: [item][contributing warp k][16 rows]
    double red[2][NWC][2];
    float redf[2][NWC][2];
    double seq_sum;                          // certified RMS fallback
    float terms[GD];
    float topw[TOPK];
    int topi[TOPK];
    uint8_t it_first[3][MAX_DN], it_kend[3][MAX_DN];   // per phase (shared, routed, down) and item:
                                                       // first contributing warp, contributors
    uint64_t full[NB];                       // chunk landed (producer arrive + bytes)
    uint64_t empty[NB];                      // chunk released (one arrival per compute warp)
    uint32_t meta[NB];                       // ring offset of a chunk in flight
    uint32_t meta_end[NB];                   // ring position after it (producer only)
    volatile int topk_ready;                 // layer + 1 whose top-8 is in topi
    volatile int abort;                      // a wait gave up: every role unwinds
    int flag;
};
static_assert(sizeof(Smem) + 128 <= 232448, "decode shared memory");
static_assert(offsetof(Smem, hid) % 16 == 0 && offsetof(Smem, u) % 16 == 0 && offsetof(Smem, tbl_r) % 16 == 0 &&
                  offsetof(Smem, tbl_d) % 16 == 0 && offsetof(Smem, ring) % 128 == 0,
              "vector-accessed shared arrays must be aligned");

__device__ __forceinline__ const uint8_t* rp(const void* base, uint64_t off) {
    return static_cast<const uint8_t*>(base) + off;
}
__device__ __forceinline__ const uint16_t* rp16(const void* base, uint64_t off) {
    return reinterpret_cast<const uint16_t*>(static_cast<const uint8_t*>(base) + off);
}
__device__ __forceinline__ int share(int n, int c, int G) { return (int)((long long)c * n / G); }

__device__ __forceinline__ void csync() { tc::named_bar_sync(1, NTC); }   // the compute warps only

__device__ __forceinline__ uint4 lds128(const void* p) { return *reinterpret_cast<const uint4*>(p); }

// ---- plan ------------------------------------------------------------------------------------------
__device__ Plan make_plan(int cta, int G) {
    Plan p;
    p.nr = cta < NE ? (NE - 1 - cta) / G + 1 : 0;
    const int S = shared_ctas(G), R = G - S;
    p.sh = cta < S;
    int n, i;
    if (p.sh) {
        p.slot = 0; p.g0 = 0; p.g1 = S;
        n = S; i = cta;
        p.t0 = share(TILES_S, i, n); p.t1 = share(TILES_S, i + 1, n);
    } else {
        int k = 0;
        while (k + 1 < TOPK && S + share(R, k + 1, TOPK) <= cta) ++k;
        p.slot = k;
        p.g0 = S + share(R, k, TOPK); p.g1 = S + share(R, k + 1, TOPK);
        n = p.g1 - p.g0; i = cta - p.g0;
        p.t0 = share(TPE, i, n); p.t1 = share(TPE, i + 1, n);
    }
    p.ot0 = share(OT, i, n); p.ot1 = share(OT, i + 1, n);
    p.n_gu = (p.t1 - p.t0 + GU_TILES - 1) / GU_TILES;
    p.dt = p.sh ? DN_TILES_S : DN_TILES_R;
    p.n_dn = (p.ot1 - p.ot0 + p.dt - 1) / p.dt;
    p.c_gu = p.nr;
    p.c_dn = p.c_gu + p.n_gu;
    p.cpl = p.c_dn + p.n_dn;
    return p;
}
__device__ __forceinline__ int dn_groups(const Plan& p) { return p.sh ? GFS : GFE; }

// Chunk i of a layer: ring bytes (copied; the allocation adds the 64-byte gate/up offset and rounds
// to 128).
__device__ uint32_t chunk_bytes(const Plan& p, int i) {
    if (i < p.c_gu) return D;
    if (i < p.c_dn) {
        const int nt = min(GU_TILES, p.t1 - p.t0 - (i - p.c_gu) * GU_TILES);
        return (uint32_t)(8 * nt) * (2 * ROW_GU + 4 * SROW_GU);
    }
    const int nt = min(p.dt, p.ot1 - p.ot0 - (i - p.c_dn) * p.dt);
    return (uint32_t)(16 * nt) * (p.sh ? DROW_S + 2 * SROW_S : DROW_R + 2 * SROW_R);
}
// Chunks stay under half the ring, so two are in flight at any ring position.
static_assert(16 * GU_TILES * 8 / 16 * (2 * ROW_GU + 4 * SROW_GU) + 192 <= RING / 2 &&
                  16 * DN_TILES_S * (DROW_S + 2 * SROW_S) + 192 <= RING / 2 &&
                  16 * DN_TILES_R * (DROW_R + 2 * SROW_R) + 192 <= RING / 2,
              "chunks fit half the ring");
static_assert((TILES_S + shared_ctas(MIN_CTAS) - 1) / shared_ctas(MIN_CTAS) <= MAX_DN &&
                  (OT + (MIN_CTAS - shared_ctas(MIN_CTAS)) / TOPK - 1) / ((MIN_CTAS - shared_ctas(MIN_CTAS)) / TOPK) <= MAX_DN,
              "per-CTA items fit the contributor tables");

// ---- mbarrier waits --------------------------------------------------------------------------------
// Bounded wait on a chunk barrier (every lane of the calling warp); false on timeout or abort.
__device__ bool wait_bar(Smem& s, const Params& P, uint64_t* bar, uint32_t parity) {
    if (tc::mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        if (tc::mbar_try_wait_sleep(bar, parity, 20000u)) return true;
        if (s.abort) return false;
        if (globaltimer_ns() - t0 > P.wait_limit_ns) {
            s.abort = 1;
            atomicExch(P.err, 1);
            atomicExch(P.sticky, 1);
            return false;
        }
    }
}
__device__ __forceinline__ bool wait_full(Smem& s, const Params& P, int c) {
    return wait_bar(s, P, &s.full[c % NB], (uint32_t)(c / NB) & 1u);
}
// This warp is done with chunks [cur, c): each is waited for (a warp that never read it still
// waits, so a released chunk has always landed) and released; then chunk c is waited for.
__device__ bool advance_to(Smem& s, const Params& P, int& cur, int c) {
    const int lane = threadIdx.x & 31;
    for (; cur < c; ++cur) {
        if (!wait_full(s, P, cur)) return false;
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&s.empty[cur % NB]);
    }
    return wait_full(s, P, c);
}
__device__ __forceinline__ bool release_to(Smem& s, const Params& P, int& cur, int c_end) {
    const int lane = threadIdx.x & 31;
    for (; cur < c_end; ++cur) {
        if (!wait_full(s, P, cur)) return false;
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&s.empty[cur % NB]);
    }
    return true;
}

// ---- producer warp ---------------------------------------------------------------------------------
// L2 prefetches (one bulk prefetch per contiguous range) of static weights whose shared-memory
// copies are issued later, so those copies read L2 instead of HBM: while the producer waits for a
// layer's top-8 it prefetches the layer's shared-down rows and the next layer's router and shared
// gate/up rows (HBM is otherwise idle until the top-8). Bulk prefetches queue in the same TMA unit
// as the copies, so none is issued after the top-8: there they delayed the routed copies.
// While a slot group's producer waits for the top-8: the next layer's router rows into L2.
__device__ void l2_static(const Plan& p, const GtmLayer* Ln, int cta, int G) {
    if (!Ln) return;
    const uint8_t* rn = static_cast<const uint8_t*>(Ln->resident_dev);
    for (int k = 0; k < p.nr; ++k) tc::prefetch_l2_bulk(rn + Ln->router.weight + (uint64_t)(cta + k * G) * D, D);
}

__device__ void producer(Smem& s, const Params& P, const Plan& p) {
    if ((threadIdx.x & 31) != 0) return;
    uint32_t head = 0, tail = 0;
    int issued = 0, released = 0;
    int expert = 0;   // the slot group's expert of the current layer
    bool ok = true;
    const int cta = blockIdx.x, G = gridDim.x;
    for (int l = 0; l < P.num_layers && ok; ++l) {
        const GtmLayer& L = P.layers[l];
        const uint8_t* res = static_cast<const uint8_t*>(L.resident_dev);
        for (int i = 0; i < p.cpl && ok; ++i) {
            if (!p.sh && i == p.c_gu) {   // the slot expert's chunks follow: wait for this layer's top-8
                l2_static(p, l + 1 < P.num_layers ? &P.layers[l + 1] : nullptr, cta, G);
                const uint64_t t0 = globaltimer_ns();
                while (s.topk_ready < l + 1) {
                    if (s.abort) { ok = false; break; }
                    if (globaltimer_ns() - t0 > P.wait_limit_ns) {
                        s.abort = 1; atomicExch(P.err, 1); atomicExch(P.sticky, 1);
                        ok = false;
                        break;
                    }
                    __nanosleep(64);
                }
                if (!ok) break;
                __threadfence_block();
                expert = s.topi[p.slot];
            }
            const uint32_t bytes = chunk_bytes(p, i);
            const uint32_t alloc = (bytes + 64 + 127) & ~127u;
            uint32_t pos = head % RING;
            if (pos + alloc > RING) { head += RING - pos; pos = 0; }
            while (head + alloc - tail > RING || issued - released >= NB) {
                // nothing in flight: the ring is empty (a skipped end of the ring counts as used
                // only while chunks issued before the skip are held)
                if (released == issued) { tail = head; break; }
                if (!wait_bar(s, P, &s.empty[released % NB], (uint32_t)(released / NB) & 1u)) { ok = false; break; }
                tail = s.meta_end[released % NB];
                ++released;
            }
            if (!ok) break;
            const int slot = issued % NB;
            s.meta[slot] = pos;
            s.meta_end[slot] = head + alloc;
            head += alloc;
            uint64_t* bar = &s.full[slot];
            uint8_t* dst = s.ring + pos;
            tc::mbar_arrive_expect_tx(bar, bytes);
            if (i < p.c_gu) {
                const int row = cta + i * G;
                tc::bulk_load(dst, res + L.router.weight + (uint64_t)row * D, D, bar);
            } else if (i < p.c_dn) {
                const int t0 = p.t0 + (i - p.c_gu) * GU_TILES, nt = min(GU_TILES, p.t1 - t0);
                const uint8_t* base = p.sh ? res : rp(L.experts_dev, (uint64_t)expert * L.expert_stride);
                const GtmQuant* qg = p.sh ? &L.shared_gate : &L.expert_gate;
                const GtmQuant* qu = p.sh ? &L.shared_up : &L.expert_up;
                const int f0 = 8 * t0;
                const uint32_t F = 8 * nt, wb = F * ROW_GU, sb = F * SROW_GU;
                tc::bulk_load(dst, base + qg->weight + (uint64_t)f0 * ROW_GU, wb, bar);
                tc::bulk_load(dst + wb + 64, base + qu->weight + (uint64_t)f0 * ROW_GU, wb, bar);
                uint8_t* sd = dst + 2 * wb + 64;
                tc::bulk_load(sd, base + qg->scales + (uint64_t)f0 * SROW_GU, sb, bar);
                tc::bulk_load(sd + sb, base + qg->biases + (uint64_t)f0 * SROW_GU, sb, bar);
                tc::bulk_load(sd + 2 * sb, base + qu->scales + (uint64_t)f0 * SROW_GU, sb, bar);
                tc::bulk_load(sd + 3 * sb, base + qu->biases + (uint64_t)f0 * SROW_GU, sb, bar);
            } else {   // down chunk j: rows of row tiles [ot0 + j dt, ...) over the whole K
                const int j = i - p.c_dn, a = p.ot0 + j * p.dt;
                const uint32_t R = 16 * min(p.dt, p.ot1 - a), r0 = 16 * a;
                const uint8_t* base = p.sh ? res : rp(L.experts_dev, (uint64_t)expert * L.expert_stride);
                const GtmQuant& q = p.sh ? L.shared_down : L.expert_down;
                const uint32_t rowb = p.sh ? DROW_S : DROW_R, srow = p.sh ? SROW_S : SROW_R;
                tc::bulk_load(dst, base + q.weight + (uint64_t)r0 * rowb, R * rowb, bar);
                tc::bulk_load(dst + R * rowb, base + q.scales + (uint64_t)r0 * srow, R * srow, bar);
                tc::bulk_load(dst + R * (rowb + srow), base + q.biases + (uint64_t)r0 * srow, R * srow, bar);
            }
            ++issued;
        }
    }
    // no exit while bulk copies into this CTA's shared memory are in flight: the chunks not yet
    // released may still be landing (released ones have been waited for by every compute warp)
    const uint64_t t0 = globaltimer_ns();
    for (int j = released; j < issued; ++j)
        while (!tc::mbar_try_wait_sleep(&s.full[j % NB], (uint32_t)(j / NB) & 1u, 20000u))
            if (globaltimer_ns() - t0 > P.wait_limit_ns) return;
}

// ---- fragment tables -----------------------------------------------------------------------------
// Table of one view (v = 0: routed_x, ab[0, D); v = 1: dense_x, ab[D, 2D)): 176 items, built by the
// compute threads from `first` on (whole warps: they take part in the builder's shuffles).
constexpr int VIEW_ITEMS = 4 * GD;
__device__ void build_views_tables(Smem& s, int first, int v) {
    constexpr int N = VIEW_ITEMS;
    const int i0 = threadIdx.x - first;
    if (i0 < 0) return;
    if (i0 < ((N + 31) & ~31)) {
        const bool on = i0 < N;
        const int k = on ? i0 : (i0 & 3), j = k >> 2, sub = k & 3;
        const float* src = s.u.t.ab + v * D + j * kGroup + 16 * sub;
        float x[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 f = reinterpret_cast<const float4*>(src)[q];
            x[4 * q] = f.x; x[4 * q + 1] = f.y; x[4 * q + 2] = f.z; x[4 * q + 3] = f.w;
        }
        uint32_t* tbl = v ? s.tbl_d : s.tbl_r;
        limb_item(x, on, tbl + (j >> 2) * QW, j & 3, sub, v ? s.gs_d : s.gs_r, j);
    }
}

// Table of the group's down inputs (written by the group's CTAs before the group barrier, read
// from L2): the shared expert's 2112 activations (33 groups, padded to 36 with zero groups) or
// the slot expert's 704 (11 groups, padded to 12).
__device__ void build_down_tables(Smem& s, const Params& P, const Plan& p) {
    const int ng = p.sh ? 4 * QSS : 4 * QS, nv = dn_groups(p), N = 4 * ng;
    const float* act = P.act + (p.sh ? 0 : FS + FE * p.slot);
    const int i0 = threadIdx.x;
    if (i0 < ((N + 31) & ~31)) {
        const bool on = i0 < N;
        const int i = on ? i0 : (i0 & 3), j = i >> 2, sub = i & 3;
        float x[16];
        if (j < nv) {
            const float4* src = reinterpret_cast<const float4*>(act + j * kGroup + 16 * sub);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float4 f = __ldcg(src + c);
                x[4 * c] = f.x; x[4 * c + 1] = f.y; x[4 * c + 2] = f.z; x[4 * c + 3] = f.w;
            }
        } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) x[e] = 0.0f;
        }
        limb_item(x, on, s.u.tbl_dn + (j >> 2) * QW, j & 3, sub, s.gs_dn, j);
    }
}

// ---- int4 tile products --------------------------------------------------------------------------
// One warp: groups [j0, j1) of a 16-row tile. ra / rb: row g / g + 8 of lane (g, t), at group 0 of
// the K range; sa, ba, sb, bb: their bf16 scales and biases at group 0; gs: per group (sum of x,
// 2^(E-6)). Lanes t = 0 and 2 accumulate groups 4Q + {0, 2} and 4Q + {1, 3} of each quad into ya
// (row g) and yb (row g + 8); the caller adds the 4 lanes of a row.
__device__ __forceinline__ void tile_groups(const uint8_t* ra, const uint8_t* rb, const uint16_t* sa, const uint16_t* ba,
                                            const uint16_t* sb, const uint16_t* bb, int j0, int j1,
                                            const uint32_t* tbl, const float2* gs, float& ya, float& yb) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const bool entry = (g & 3) < 3 && (g >> 2) == (t >> 1);
    const int e = 6 * (t >> 1) + 2 * (g & 3) + (t & 1);
    for (int Q = j0 >> 2; Q * 4 < j1; ++Q) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int j = 4 * Q + 2 * h + (t >> 1);   // the group of this lane's K slots and B entry
            if (4 * Q + 2 * h + 1 < j0 || 4 * Q + 2 * h >= j1) continue;   // warp-uniform
            const uint4 wa = lds128(ra + 128 * Q + 64 * h + 16 * t);
            const uint4 wb = lds128(rb + 128 * Q + 64 * h + 16 * t);
            uint4 b01 = make_uint4(0u, 0u, 0u, 0u), b23 = b01;
            if (entry && j >= j0 && j < j1) {
                const uint32_t* ep = tbl + (2 * Q + h) * 96 + e * 8;
                b01 = lds128(ep);
                b23 = lds128(ep + 4);
            }
            const uint32_t wA[4] = {wa.x, wa.y, wa.z, wa.w}, wB[4] = {wb.x, wb.y, wb.z, wb.w};
            const uint32_t bw[8] = {b01.x, b01.y, b01.z, b01.w, b23.x, b23.y, b23.z, b23.w};
            int d[4] = {0, 0, 0, 0};
#pragma unroll
            for (int w = 0; w < 4; ++w)
                mma_u8s8(d, wA[w] & 0x0F0F0F0Fu, wB[w] & 0x0F0F0F0Fu, (wA[w] >> 4) & 0x0F0F0F0Fu, (wB[w] >> 4) & 0x0F0F0F0Fu,
                         bw[2 * w], bw[2 * w + 1]);
            // columns 2t, 2t + 1: lane t even holds limbs 0, 1 of its group, t odd limb 2 (and a zero column)
            float pa = (t & 1) ? (float)d[0] * 6.103515625e-05f : fmaf((float)d[1], 0.0078125f, (float)d[0]);
            float pb = (t & 1) ? (float)d[2] * 6.103515625e-05f : fmaf((float)d[3], 0.0078125f, (float)d[2]);
            pa += __shfl_xor_sync(0xffffffffu, pa, 1);
            pb += __shfl_xor_sync(0xffffffffu, pb, 1);
            if (!(t & 1) && j >= j0 && j < j1) {
                const float2 gj = gs[j];
                ya = fmaf(bf16f(ba[j]), gj.x, fmaf(bf16f(sa[j]) * gj.y, pa, ya));
                yb = fmaf(bf16f(bb[j]), gj.x, fmaf(bf16f(sb[j]) * gj.y, pb, yb));
            }
        }
    }
}

// The warps' split of n_items x L (item, group) pairs: warp w takes pairs [pw0(w), pw0(w + 1)).
__device__ __forceinline__ int pw0(int w, int total) { return w * total / NWC; }   // total <= 1024

// Warps that work on item i: from the last warp whose range starts at or before pair i L, i.e.
// ceil((i L + 1) NWC / total) - 1, to the one holding pair (i + 1) L - 1. A warp's range holds at
// least floor(total / NWC) pairs, so at most max_k = ceil((L - 1) / floor(total / NWC)) + 1 warps
// share an item; warp w keeps its partial of item i in slot [(i max_k + w - first(i)) 16 + row].
struct Split {
    int total, max_k;
};
__device__ __forceinline__ Split make_split(int n, int L) {
    Split sp;
    sp.total = n * L;
    const int ppw = sp.total / NWC;
    sp.max_k = ppw > 0 ? (L - 1 + ppw - 1) / ppw + 1 : NWC;
    return sp;
}
__device__ __forceinline__ int first_warp(const Split& sp, int i, int L) {
    return ((i * L + 1) * NWC + sp.total - 1) / sp.total - 1;
}
// The contributor table of one phase (ph: 0 shared gate/up, 1 routed gate/up, 2 down), once per
// launch by one thread.
__device__ void fill_items(Smem& s, int ph, int n, int L) {
    if (n <= 0) return;
    const Split sp = make_split(n, L);
    for (int i = 0; i < n; ++i) {
        const int f = first_warp(sp, i, L);
        const int last = min(NWC - 1, ((i + 1) * L * NWC + sp.total - 1) / sp.total - 1);   // holds pair (i + 1) L - 1
        s.it_first[ph][i] = (uint8_t)f;
        s.it_kend[ph][i] = (uint8_t)(last - f + 1);
    }
}
// Sum of item i's partials for tile row r, in warp order.
__device__ __forceinline__ float item_sum(const Smem& s, const Split& sp, int ph, int i, int r) {
    const float* p = s.slot + (i * sp.max_k) * 16 + r;
    const int k_end = s.it_kend[ph][i];
    float v = 0.0f;
    for (int k = 0; k < k_end; ++k) v += p[16 * k];
    return v;
}
__device__ __forceinline__ float* slot_of(Smem& s, const Split& sp, int ph, int i, int warp) {
    return s.slot + (i * sp.max_k + warp - s.it_first[ph][i]) * 16;
}

// Source rows of one 16-row tile for tile_groups.
struct TileSrc {
    const uint8_t* ra; const uint8_t* rb;
    const uint16_t* sa; const uint16_t* ba; const uint16_t* sb; const uint16_t* bb;
    const uint32_t* tbl; const float2* gs;
};

// Gate/up tile lt of a chunk of F features per matrix at `base`: rows 0-3 gate f0..3, 4-7 up f0..3,
// 8-11 gate f0+4..7, 12-15 up f0+4..7 (f0 = 8 lt within the chunk).
__device__ __forceinline__ TileSrc gu_src(const uint8_t* base, int F, int lt, const uint32_t* tbl, const float2* gs) {
    const int g = (threadIdx.x & 31) >> 2;
    const bool up = g >= 4;
    const int r = 8 * lt + (g & 3);
    const uint32_t wb = (uint32_t)F * ROW_GU, sbytes = (uint32_t)F * SROW_GU;
    const uint8_t* w = base + (up ? wb + 64 : 0);
    const uint8_t* sc = base + 2 * wb + 64 + (up ? 2 * sbytes : 0);
    TileSrc S;
    S.ra = w + (uint32_t)r * ROW_GU;
    S.rb = S.ra + 4 * ROW_GU;
    S.sa = reinterpret_cast<const uint16_t*>(sc) + r * GD;
    S.ba = reinterpret_cast<const uint16_t*>(sc + sbytes) + r * GD;
    S.sb = S.sa + 4 * GD;
    S.bb = S.ba + 4 * GD;
    S.tbl = tbl; S.gs = gs;
    return S;
}

// One phase of gate/up tiles [t_first, t_first + n): locate(tile) gives (chunk index c, first tile of
// the chunk, tiles in the chunk). Every warp works its pairs, then releases the phase's chunks
// [c_begin, c_end). Returns false when a wait gave up.
template <class Locate>
__device__ bool gu_phase(Smem& s, const Params& P, int ph, int n, int c_begin, int c_end, const uint32_t* tbl,
                         const float2* gs, Locate locate) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const Split sp = make_split(n, GD);
    int p = pw0(warp, sp.total);
    const int p1 = pw0(warp + 1, sp.total);
    int cur = c_begin;
    bool ok = true;
    while (p < p1) {
        const int item = p / GD, j0 = p - item * GD, j1 = min(GD, j0 + (p1 - p));
        int c, lt, F;
        locate(item, c, lt, F);
        if (!advance_to(s, P, cur, c)) { ok = false; break; }
        const TileSrc S = gu_src(s.ring + s.meta[c % NB], F, lt, tbl, gs);
        float ya = 0.0f, yb = 0.0f;
        tile_groups(S.ra, S.rb, S.sa, S.ba, S.sb, S.bb, j0, j1, S.tbl, S.gs, ya, yb);
        ya += __shfl_xor_sync(0xffffffffu, ya, 1);
        ya += __shfl_xor_sync(0xffffffffu, ya, 2);
        yb += __shfl_xor_sync(0xffffffffu, yb, 1);
        yb += __shfl_xor_sync(0xffffffffu, yb, 2);
        if (t == 0) {
            float* sl = slot_of(s, sp, ph, item, warp);
            sl[g] = ya;
            sl[8 + g] = yb;
        }
        p += j1 - j0;
    }
    if (ok) ok = release_to(s, P, cur, c_end);
    return ok;
}

__device__ __forceinline__ float gelu_tanh_f(float x) {
    return 0.5f * x * (1.0f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
}

// GeGLU of the phase's n tiles -> act[off + 8 * (first + item) + f].
__device__ void gu_epilogue(const Smem& s, int ph, float* act, int n) {
    const Split sp = make_split(n, GD);
    for (int i = threadIdx.x; i < n * 8; i += NTC) {
        const int item = i >> 3, f = i & 7;
        const int rg = (f & 3) + 8 * (f >> 2);
        const float gt = item_sum(s, sp, ph, item, rg), up = item_sum(s, sp, ph, item, rg + 4);
        act[8 * item + f] = gelu_tanh_f(gt) * up;
    }
}

// ---- barriers ----------------------------------------------------------------------------------
// The CTA's writes before the barrier are ordered before the flag by the release store (its fence
// is cumulative over the writes the barrier made visible to thread 0).
__device__ __forceinline__ void arrive(const Params& P, unsigned* flags, unsigned value) {
    csync();
    if (threadIdx.x == 0) st_release(flags + blockIdx.x, value);
}

// Warp 0 polls the flags of CTAs [lo, hi); the other compute warps wait at the named barrier.
__device__ bool wait_range(Smem& s, const Params& P, const unsigned* f, int lo, int hi, unsigned value) {
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        const uint64_t t0 = globaltimer_ns();
        bool ok = true;
        for (;;) {
            bool mine = true;
            for (int b = lo + lane; b < hi; b += 32) mine &= (ld_relaxed(f + b) >= value);
            const int e = lane == 0 ? ld_volatile_int(P.err) : 0;
            if (__all_sync(0xffffffffu, mine)) break;
            if (__shfl_sync(0xffffffffu, e, 0) != 0) { ok = false; break; }
            if (globaltimer_ns() - t0 > P.wait_limit_ns) {
                if (lane == 0) { atomicExch(P.err, 1); atomicExch(P.sticky, 1); }
                ok = false;
                break;
            }
        }
        __threadfence();
        if (lane == 0) { s.flag = ok ? 0 : 1; if (!ok) s.abort = 1; }
    }
    csync();
    return s.flag == 0;
}
__device__ __forceinline__ bool wait_all(Smem& s, const Params& P, const unsigned* f, unsigned value) {
    return wait_range(s, P, f, 0, (int)gridDim.x, value);
}

__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// A logit word carries its own payload (layer number and value in one 64-bit store), so it needs
// no release ordering.
__device__ __forceinline__ void st_relaxed_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" :: "l"(p), "l"(v) : "memory");
}

// ---- layer tail and views --------------------------------------------------------------------------
// Norm vectors of one compute thread's four elements (4 bf16 each), loaded before the tail's wait.
struct Norms {
    uint2 w1, w2, w3;       // post_ffn_norm_1, post_ffn_norm_2, post_ffn_norm of the previous layer
    uint2 pre, pre2, rsc;   // pre_ffn_norm, pre_ffn_norm_2, router.scale of this layer
    float ls;               // layer_scalar of the previous layer
};
__device__ __forceinline__ uint2 ldg_u2(const void* base, uint64_t off, int i) {
    return __ldg(reinterpret_cast<const uint2*>(rp(base, off)) + i);
}
__device__ Norms load_norms(const GtmLayer* Lp, const GtmLayer* L) {
    Norms n;
    const int i = threadIdx.x;
    n.w1 = n.w2 = n.w3 = n.pre = n.pre2 = n.rsc = make_uint2(0u, 0u);
    n.ls = 0.0f;
    if (Lp) {
        n.w1 = ldg_u2(Lp->resident_dev, Lp->post_ffn_norm_1, i);
        n.w2 = ldg_u2(Lp->resident_dev, Lp->post_ffn_norm_2, i);
        n.w3 = ldg_u2(Lp->resident_dev, Lp->post_ffn_norm, i);
        n.ls = bf16f(__ldg(rp16(Lp->resident_dev, Lp->layer_scalar)));
    }
    if (L) {
        n.pre = ldg_u2(L->resident_dev, L->pre_ffn_norm, i);
        n.pre2 = ldg_u2(L->resident_dev, L->pre_ffn_norm_2, i);
        n.rsc = ldg_u2(L->resident_dev, L->router_scale, i);
    }
    return n;
}
__device__ __forceinline__ float bfw(const uint2& v, int k) {   // element k (0..3) of 4 packed bf16
    const uint32_t w = k < 2 ? v.x : v.y;
    return bf16f((uint16_t)((k & 1) ? (w >> 16) : (w & 0xFFFFu)));
}

// Sums a and b over the compute threads with one barrier: every thread adds the warp partials itself
// in warp order, so every thread (and every CTA, given the same data) gets the same bits.
// Consecutive calls must alternate `buf`.
__device__ __forceinline__ double2 block_sum2(Smem& s, double a, double b, int buf) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        a += __shfl_xor_sync(0xffffffffu, a, o);
        b += __shfl_xor_sync(0xffffffffu, b, o);
    }
    if (lane == 0) { s.red[buf][warp][0] = a; s.red[buf][warp][1] = b; }
    csync();
    double ra[4] = {0.0, 0.0, 0.0, 0.0}, rb[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll
    for (int w = 0; w < NWC; ++w) { ra[w & 3] += s.red[buf][w][0]; rb[w & 3] += s.red[buf][w][1]; }
    return make_double2((ra[0] + ra[1]) + (ra[2] + ra[3]), (rb[0] + rb[1]) + (rb[2] + rb[3]));
}

// The same in float, for the tail's norms (not the exact one of the views): about 1e-7 relative.
__device__ __forceinline__ float2 block_sum2f(Smem& s, float a, float b, int buf) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        a += __shfl_xor_sync(0xffffffffu, a, o);
        b += __shfl_xor_sync(0xffffffffu, b, o);
    }
    if (lane == 0) { s.redf[buf][warp][0] = a; s.redf[buf][warp][1] = b; }
    csync();
    float ra[4] = {0.0f, 0.0f, 0.0f, 0.0f}, rb[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int w = 0; w < NWC; ++w) { ra[w & 3] += s.redf[buf][w][0]; rb[w & 3] += s.redf[buf][w][1]; }
    return make_float2((ra[0] + ra[1]) + (ra[2] + ra[3]), (rb[0] + rb[1]) + (rb[2] + rb[3]));
}

// 1 / sqrt(float(sum / D) + eps), the reference's formula (src/cpu_reference.cpp:46), from a float
// sum of squares; the mean is formed with a multiply by 1/D.
constexpr double kInvD = 1.0 / (double)D;
__device__ __forceinline__ float rms_inv_from_sumf(float sum, float eps) {
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(sum * (1.0f / (float)D), eps)));
}
__device__ __forceinline__ float sq4f(const float (&v)[4]) {
    return fmaf(v[0], v[0], fmaf(v[1], v[1], fmaf(v[2], v[2], v[3] * v[3])));
}

// The same with the reference's exact bits when `sum` is a parallel double sum of x*x: see
// exact_rms_inv for the argument; the bound (D + 48) ulps also covers the tree depth (< 30) and
// the multiply by the rounded 1/D. The check is identical on every thread, so the rare fallback
// (a sequential sum by thread 0, then the reference's division) is a uniform branch.
__device__ float certified_rms_inv(Smem& s, const float* x, double sum, float eps) {
    const double q = __dmul_rn(sum, kInvD);
    float f = __double2float_rn(q);
    const double fd = (double)f;
    const double lo = (fd + (double)nextafterf(f, -INFINITY)) * 0.5;
    const double hi = (fd + (double)nextafterf(f, INFINITY)) * 0.5;
    const double bound = q * ((double)D + 48.0) * 1.1102230246251565e-16;
    if (!(q - lo > bound && hi - q > bound)) {
        if (threadIdx.x == 0) {
            double seq = 0.0;
            for (int i = 0; i < D; ++i) seq = __dadd_rn(seq, __dmul_rn((double)x[i], (double)x[i]));
            s.seq_sum = seq;
        }
        csync();
        f = __double2float_rn(__ddiv_rn(s.seq_sum, (double)D));
    }
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(f, eps)));
}

__device__ __forceinline__ double sq4(const float (&v)[4]) {
    return (double)v[0] * v[0] + (double)v[1] * v[1] + (double)v[2] * v[2] + (double)v[3] * v[3];
}

// Layer tail of the previous layer (src/cpu_reference.cpp:512-520), when there is one, from the down
// partials (shared output = the 3 shared thirds, h2 = the 8 routed experts in router order), the
// optional weightless RMSNorm between layers, then the views of this layer
// (src/cpu_reference.cpp:425-443): dense_x = h*w_pre, routed_x = h*w_pre2 and
// router_in = h*bf16(router.scale)*(1/sqrt(D)) with h = rmsnorm_no_scale(hidden), exactly as the
// reference rounds them (their fragment tables are built next to the router rows). Compute thread
// i owns elements 4i..4i+3.
__device__ void tail_and_views(Smem& s, const Params& P, const Norms& nv, bool has_prev, bool norm_between,
                               bool do_views, float* h1_out, float* h2_out, float* hid_out) {
    const int i = threadIdx.x;
    float hv[4];
    {
        const float4 v = reinterpret_cast<const float4*>(s.hid)[i];
        hv[0] = v.x; hv[1] = v.y; hv[2] = v.z; hv[3] = v.w;
    }
    int buf = 0;
    if (has_prev) {
        // part [1 + TOPK][D]: the shared down row, then the slots' rows; h2 = sum_k w_k out_k in
        // router order (src/cpu_reference.cpp:508-509), each product rounded
        const float4* pp = reinterpret_cast<const float4*>(P.part);
        float4 pr[TOPK];
        const float4 ps = __ldcg(pp + i);
#pragma unroll
        for (int k = 0; k < TOPK; ++k) pr[k] = __ldcg(pp + (1 + k) * (D / 4) + i);
        float sh[4] = {ps.x, ps.y, ps.z, ps.w};
        float h2[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int k = 0; k < TOPK; ++k) {
            const float w = s.topw[k];
            h2[0] = __fadd_rn(h2[0], __fmul_rn(w, pr[k].x));
            h2[1] = __fadd_rn(h2[1], __fmul_rn(w, pr[k].y));
            h2[2] = __fadd_rn(h2[2], __fmul_rn(w, pr[k].z));
            h2[3] = __fadd_rn(h2[3], __fmul_rn(w, pr[k].w));
        }
        float2 r = block_sum2f(s, sq4f(sh), sq4f(h2), buf); buf ^= 1;
        const float inv1 = rms_inv_from_sumf(r.x, P.eps), inv2 = rms_inv_from_sumf(r.y, P.eps);
        float tt[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float h1 = __fmul_rn(__fmul_rn(sh[k], inv1), bfw(nv.w1, k));
            tt[k] = __fadd_rn(__fmul_rn(__fmul_rn(h2[k], inv2), bfw(nv.w2, k)), h1);
            sh[k] = h1;
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {   // caller buffers: scalar stores (4-byte alignment is all they promise)
            if (h1_out) h1_out[4 * i + k] = sh[k];
            if (h2_out) h2_out[4 * i + k] = h2[k];
        }
        r = block_sum2f(s, sq4f(tt), 0.0f, buf); buf ^= 1;
        const float inv3 = rms_inv_from_sumf(r.x, P.eps);
#pragma unroll
        for (int k = 0; k < 4; ++k)
            hv[k] = __fmul_rn(__fadd_rn(hv[k], __fmul_rn(__fmul_rn(tt[k], inv3), bfw(nv.w3, k))), nv.ls);
        if (norm_between) {
            r = block_sum2f(s, sq4f(hv), 0.0f, buf); buf ^= 1;
            const float inv4 = rms_inv_from_sumf(r.x, P.eps);
#pragma unroll
            for (int k = 0; k < 4; ++k) hv[k] = __fmul_rn(hv[k], inv4);
        }
        reinterpret_cast<float4*>(s.hid)[i] = make_float4(hv[0], hv[1], hv[2], hv[3]);
        if (hid_out)
#pragma unroll
            for (int k = 0; k < 4; ++k) hid_out[4 * i + k] = hv[k];
    }
    if (!do_views) {
        csync();
        return;
    }
    const double2 r = block_sum2(s, sq4(hv), 0.0, buf);   // its barrier also publishes s.hid
    const float inv = certified_rms_inv(s, s.hid, r.x, P.eps);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int e = 4 * i + k;
        const float h = __fmul_rn(hv[k], inv);
        s.u.t.ab[D + e] = __fmul_rn(h, bfw(nv.pre, k));    // dense_x
        s.u.t.ab[e] = __fmul_rn(h, bfw(nv.pre2, k));       // routed_x
        s.u.t.rin[(e >> 6) * RIN_PITCH + (e & 63)] = __fmul_rn(__fmul_rn(h, bfw(nv.rsc, k)), P.inv_sqrt_d);
    }
    csync();
}

// One router logit in src/cpu_reference.cpp:86-106's order (bit-identical), row weights in `W`
// (shared memory); threads 0..43 take a group each (their scale and bias already loaded), thread 0
// adds the 44 terms in order. Called by the first two compute warps.
__device__ float router_row(Smem& s, const uint8_t* W, float sc, float bi) {
    const int tid = threadIdx.x;
    if (tid < GD) {
        const uint4* wg = reinterpret_cast<const uint4*>(W + tid * kGroup);
        uint4 q[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) q[i] = wg[i];
        const float* x = s.u.t.rin + tid * RIN_PITCH;
        float dot = 0.0f, sum = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t wv[4] = {q[i].x, q[i].y, q[i].z, q[i].w};
#pragma unroll
            for (int c = 0; c < 4; ++c) {
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const float xv = x[i * 16 + c * 4 + b];
                    dot = __fadd_rn(dot, __fmul_rn((float)((wv[c] >> (8 * b)) & 0xFFu), xv));
                    sum = __fadd_rn(sum, xv);
                }
            }
        }
        s.terms[tid] = __fadd_rn(__fmul_rn(sc, dot), __fmul_rn(bi, sum));
    }
    tc::named_bar_sync(2, 64);
    float acc = 0.0f;
    if (tid == 0)
        for (int g = 0; g < GD; ++g) acc = __fadd_rn(acc, s.terms[g]);
    return acc;
}

// Top-8 of the 128 logits (lane j of warp 0 holds rows j + 32 k) by (value desc, index asc),
// softmax over the 8, times per_expert_scale (src/cpu_reference.cpp:447-480); pes_w holds the
// per-expert scales of the same rows. Results in s.topi / s.topw.
__device__ void select_topk(Smem& s, const float (&v)[4], const uint16_t (&pes_w)[4], bool writer, uint32_t* idx_out,
                            float* w_out, float* logits_out) {
    const int lane = threadIdx.x;
    bool taken[4] = {false, false, false, false};
    if (writer && logits_out)
#pragma unroll
        for (int j = 0; j < 4; ++j) logits_out[lane + 32 * j] = v[j];
    // order-preserving unsigned keys (-0 folded onto +0, which compare equal as floats); each
    // round takes the largest key, then the lowest index holding it: (value desc, index asc)
    uint32_t key[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t u = __float_as_uint(v[j] == 0.0f ? 0.0f : v[j]);
        key[j] = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    }
    float my_sel = 0.0f, top0 = 0.0f;
    int my_idx = 0;
#pragma unroll
    for (int k = 0; k < TOPK; ++k) {
        uint32_t ck = 0u, ci = 0xFFFFFFFFu;          // this lane's best untaken (key desc, index asc)
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (!taken[j] && (ci == 0xFFFFFFFFu || key[j] > ck)) { ck = key[j]; ci = (uint32_t)(lane + 32 * j); }
        const uint32_t mk = __reduce_max_sync(0xffffffffu, ck);
        const uint32_t bi = __reduce_min_sync(0xffffffffu, ck == mk ? ci : 0xFFFFFFFFu);
        const float bv = __uint_as_float((mk & 0x80000000u) ? (mk & 0x7FFFFFFFu) : ~mk);
        if (k == 0) top0 = bv;
        if (lane == k) { my_sel = bv; my_idx = (int)bi; }
#pragma unroll
        for (int j = 0; j < 4; ++j) if ((uint32_t)(lane + 32 * j) == bi) taken[j] = true;
    }
    // the selected rows' per-expert scales from the lanes holding them
    uint16_t pes_bits = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint16_t pv = (uint16_t)__shfl_sync(0xffffffffu, (int)pes_w[j], my_idx & 31);
        if ((my_idx >> 5) == j) pes_bits = pv;
    }
    // lanes 0..7: exp in parallel, the sum in order on every lane
    const float e = lane < TOPK ? expf(__fsub_rn(my_sel, top0)) : 0.0f;
    float sum = 0.0f;
#pragma unroll
    for (int k = 0; k < TOPK; ++k) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, e, k));
    if (lane < TOPK) {
        const float w = __fmul_rn(__fdiv_rn(e, sum), bf16f(pes_bits));
        s.topi[lane] = my_idx;
        s.topw[lane] = w;
        if (writer && idx_out) idx_out[lane] = (uint32_t)my_idx;
        if (writer && w_out) w_out[lane] = w;
    }
}

// ---- down phase ------------------------------------------------------------------------------------
// Contributor tables of the CTA's gate/up tiles and down row tiles, once per launch.
__device__ void plan_items(Smem& s, const Plan& p) {
    if (threadIdx.x != 0) return;
    fill_items(s, p.sh ? 0 : 1, p.t1 - p.t0, GD);
    fill_items(s, 2, p.ot1 - p.ot0, dn_groups(p));
}

// The CTA's down row tiles [ot0, ot1) over the whole K of its expert (33 or 11 groups) from the
// down chunks c, c + 1, ... (dt row tiles each): n row tiles x groups pairs split over the warps.
__device__ bool down_phase(Smem& s, const Params& P, const Plan& p, int c) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int Lg = dn_groups(p), n = p.ot1 - p.ot0;
    const Split sp = make_split(n, Lg);
    int pp = pw0(warp, sp.total);
    const int p1 = pw0(warp + 1, sp.total);
    int cur = c;
    bool ok = true;
    const int rowb = p.sh ? DROW_S : DROW_R;
    while (pp < p1) {
        const int k = pp / Lg, j0 = pp - k * Lg, j1 = min(Lg, j0 + (p1 - pp));
        const int ck = k / p.dt, R = 16 * min(p.dt, n - ck * p.dt);   // its chunk, rows in the chunk
        if (!advance_to(s, P, cur, c + ck)) { ok = false; break; }
        const uint8_t* base = s.ring + s.meta[(c + ck) % NB];
        const int row = 16 * (k - ck * p.dt) + g;
        const uint8_t* w = base + (uint32_t)row * rowb;
        const uint16_t* sc = reinterpret_cast<const uint16_t*>(base + (uint32_t)R * rowb) + row * Lg;
        const uint16_t* bi = sc + R * Lg;
        float ya = 0.0f, yb = 0.0f;
        tile_groups(w, w + 8 * rowb, sc, bi, sc + 8 * Lg, bi + 8 * Lg, j0, j1, s.u.tbl_dn, s.gs_dn, ya, yb);
        ya += __shfl_xor_sync(0xffffffffu, ya, 1);
        ya += __shfl_xor_sync(0xffffffffu, ya, 2);
        yb += __shfl_xor_sync(0xffffffffu, yb, 1);
        yb += __shfl_xor_sync(0xffffffffu, yb, 2);
        if (t == 0) {
            float* sl = slot_of(s, sp, 2, k, warp);
            sl[g] = ya;
            sl[8 + g] = yb;
        }
        pp += j1 - j0;
    }
    if (ok) ok = release_to(s, P, cur, c + p.n_dn);
    return ok;
}

// The CTA's down rows (each row whole: its warps' partials summed in warp order) into the shared
// row of part, or the slot's (the tail weights and sums the slots in router order).
__device__ void down_epilogue(Smem& s, const Params& P, const Plan& p) {
    const int n = p.ot1 - p.ot0;
    const Split sp = make_split(n, dn_groups(p));
    float* dst = P.part + (p.sh ? 0 : (size_t)(1 + p.slot) * D) + 16 * p.ot0;
    for (int i = threadIdx.x; i < n * 16; i += NTC) dst[i] = item_sum(s, sp, 2, i >> 4, i & 15);
}

// Wait for all 128 logit words of layer l (warp 0), then the top-8 (topi, topw; the writer's outputs).
__device__ bool topk_step(Smem& s, const Params& P, int l, unsigned ep, const uint16_t (&pes_w)[4], bool writer) {
    const GtmDecodeIO& io = P.io;
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        const unsigned want = ep + (l == 0 ? P.first_wait_extra : 0u);
        float v[4];
        const uint64_t t0 = globaltimer_ns();
        bool wok = true;
        for (;;) {
            bool mine = true;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const unsigned long long w = ld_relaxed_u64(P.logit_words + lane + 32 * j);
                mine &= (unsigned)(w >> 32) >= want;
                v[j] = __uint_as_float((uint32_t)w);
            }
            const int e = lane == 0 ? ld_volatile_int(P.err) : 0;
            if (__all_sync(0xffffffffu, mine)) break;
            if (__shfl_sync(0xffffffffu, e, 0) != 0) { wok = false; break; }
            if (globaltimer_ns() - t0 > P.wait_limit_ns) {
                if (lane == 0) { atomicExch(P.err, 1); atomicExch(P.sticky, 1); }
                wok = false;
                break;
            }
        }
        __threadfence();
        if (wok) {
            select_topk(s, v, pes_w, writer, io.topk_idx_dev ? io.topk_idx_dev + (size_t)l * TOPK : nullptr,
                        io.topk_w_dev ? io.topk_w_dev + (size_t)l * TOPK : nullptr,
                        io.logits_dev ? io.logits_dev + (size_t)l * NE : nullptr);
            __syncwarp();
            __threadfence_block();
            if (lane == 0) s.topk_ready = l + 1;
        } else if (lane == 0) {
            s.abort = 1;
        }
    }
    csync();
    return !s.abort;
}

// ---- the kernel --------------------------------------------------------------------------------------
__global__ void __launch_bounds__(NT, 1) moe_decode_kernel(const __grid_constant__ Params P) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    const GtmDecodeIO& io = P.io;
    const bool writer = cta == 0;
    const Plan p = make_plan(cta, G);

    if (tid == 0) {
        for (int b = 0; b < NB; ++b) { tc::mbar_init(&s.full[b], 1); tc::mbar_init(&s.empty[b], NWC); }
        s.topk_ready = 0;
        s.abort = 0;
        tc::mbar_fence_init();
    }
    plan_items(s, p);
    __syncthreads();
    if (warp == NWC) {
        producer(s, P, p);
        return;
    }

    for (int i = tid; i < D; i += NTC) s.hid[i] = io.hidden_in_dev[i];
    csync();
    const bool norm_between = (io.flags & GTM_DECODE_NORM_BETWEEN_LAYERS) != 0;
    int cbase = 0;   // chunk sequence number of the layer's first chunk
    for (int l = 0; l < P.num_layers; ++l, cbase += p.cpl) {
        const GtmLayer& L = P.layers[l];
        const GtmLayer* Lp = l > 0 ? &P.layers[l - 1] : nullptr;
        const unsigned ep = (unsigned)(l + 1);
        // loads that need no barrier: the norm vectors of the tail and views, this CTA's router
        // scale and bias (first row), the per-expert scales for the top-8
        const Norms nv = load_norms(Lp, &L);
        float rsc = 0.0f, rbi = 0.0f;
        if (tid < GD && p.nr > 0) {
            rsc = bf16f(__ldg(rp16(L.resident_dev, L.router.scales) + cta * GD + tid));
            rbi = bf16f(__ldg(rp16(L.resident_dev, L.router.biases) + cta * GD + tid));
        }
        uint16_t pes_w[4] = {0, 0, 0, 0};
        if (warp == 0)
#pragma unroll
            for (int j = 0; j < 4; ++j) pes_w[j] = __ldg(rp16(L.resident_dev, L.per_expert_scale) + lane + 32 * j);

        // ---- tail + views ----
        if (l > 0 && !wait_all(s, P, P.flags_c, ep - 1)) break;
        tail_and_views(s, P, nv, l > 0, norm_between, true,
                       writer && io.h1_dev && l > 0 ? io.h1_dev + (size_t)(l - 1) * D : nullptr,
                       writer && io.h2_dev && l > 0 ? io.h2_dev + (size_t)(l - 1) * D : nullptr,
                       writer && io.hidden_layers_dev && l > 0 ? io.hidden_layers_dev + (size_t)(l - 1) * D : nullptr);

        // ---- router rows (the logit words double as barrier A) on warps 0-1, while warps 2-7
        //      build the fragment table of the group's view ----
        int cur = cbase;
        bool ok = true;
        if (warp >= 2) build_views_tables(s, 64, p.sh ? 1 : 0);
        for (int k = 0; k < p.nr; ++k) {
            if (warp < 2) {
                const int row = cta + k * G;
                if (!advance_to(s, P, cur, cbase + k)) ok = false;
                if (k > 0 && tid < GD) {
                    rsc = bf16f(__ldg(rp16(L.resident_dev, L.router.scales) + row * GD + tid));
                    rbi = bf16f(__ldg(rp16(L.resident_dev, L.router.biases) + row * GD + tid));
                }
                float lg = router_row(s, s.ring + s.meta[(cbase + k) % NB], rsc, rbi);
                if (tid == 0 && ok) {
                    if (io.logit_bias_dev) lg = __fadd_rn(lg, io.logit_bias_dev[(size_t)l * NE + row]);
                    st_relaxed_u64(P.logit_words + row, ((unsigned long long)ep << 32) | __float_as_uint(lg));
                }
                tc::named_bar_sync(2, 64);   // the row's words are read before the chunk is released
            }
        }
        if (ok) ok = release_to(s, P, cur, cbase + p.nr);
        if (!ok) s.abort = 1;
        csync();   // the view table is complete
        if (s.abort) break;

        // the slot groups need the top-8 first; the shared group takes it after its down rows
        // (every logit word of the layer is out by then, and none is overwritten before barrier C)
        if (!p.sh && !topk_step(s, P, l, ep, pes_w, writer)) break;

        // ---- the group expert's gate/up tiles ----
        const int ph = p.sh ? 0 : 1;
        ok = gu_phase(s, P, ph, p.t1 - p.t0, cbase + p.c_gu, cbase + p.c_dn, p.sh ? s.tbl_d : s.tbl_r,
                      p.sh ? s.gs_d : s.gs_r, [&](int item, int& c, int& lt, int& F) {
                          const int k = item / GU_TILES;
                          c = cbase + p.c_gu + k;
                          lt = item - k * GU_TILES;
                          F = 8 * min(GU_TILES, p.t1 - p.t0 - k * GU_TILES);
                      });
        if (!ok) s.abort = 1;
        csync();
        if (s.abort) break;
        gu_epilogue(s, ph, P.act + (p.sh ? 0 : FS + FE * p.slot) + 8 * p.t0, p.t1 - p.t0);

        // ---- the group barrier: every activation of the group's expert ----
        arrive(P, P.flags_b, ep);
        if (!wait_range(s, P, P.flags_b, p.g0, p.g1, ep)) break;

        // ---- the expert's down rows [16 ot0, 16 ot1) ----
        build_down_tables(s, P, p);
        csync();
        ok = down_phase(s, P, p, cbase + p.c_dn);
        if (!ok) s.abort = 1;
        csync();
        if (s.abort) break;
        down_epilogue(s, P, p);
        if (p.sh && !topk_step(s, P, l, ep, pes_w, writer)) break;
        arrive(P, P.flags_c, ep);
    }
    csync();
    if (s.abort) return;

    // final tail by CTA 0
    if (!writer) return;
    const int l = P.num_layers;
    const Norms nv = load_norms(&P.layers[l - 1], nullptr);
    if (!wait_all(s, P, P.flags_c, (unsigned)l)) return;
    tail_and_views(s, P, nv, true, false, false, io.h1_dev ? io.h1_dev + (size_t)(l - 1) * D : nullptr,
                   io.h2_dev ? io.h2_dev + (size_t)(l - 1) * D : nullptr,
                   io.hidden_layers_dev ? io.hidden_layers_dev + (size_t)(l - 1) * D : nullptr);
    csync();
    for (int i = tid; i < D; i += NTC) io.hidden_out_dev[i] = s.hid[i];
}

}  // namespace dec

// Workspace: [0, 1024) the 128 router logit words, [2048, 3072) barrier-B flags, [3072, 4096)
// barrier-C flags and [4096] this launch's error word, all cleared before every launch; [4100] the
// sticky error word (zero-initialised once by the workspace's owner, read and cleared by
// gtm_moe_decode_check); from 4352: activations and down partials.
constexpr size_t kErrOffset = 4096, kStickyOffset = 4100, kDataOffset = 4352;

size_t decode_workspace_bytes() {
    return kDataOffset + sizeof(float) * (dec::ACT_R + dec::FS + (size_t)(1 + dec::TOPK) * dec::D) + 256;
}
size_t decode_sticky_offset() { return kStickyOffset; }

int launch_decode(const GtmDims& dims, const GtmLayer* layers, int num_layers, const GtmDecodeIO& io,
                  void* ws, size_t ws_bytes, cudaStream_t stream, int num_ctas) {
    using namespace dec;
    (void)ws_bytes;
    if (num_ctas < MIN_CTAS || num_ctas > MAX_CTAS)
        return set_error(GTM_ERR_UNSUPPORTED, "gtm_moe_decode: %d CTAs outside the decode's work split", num_ctas);
    Params P;
    memset(&P, 0, sizeof(P));
    for (int l = 0; l < num_layers; ++l) P.layers[l] = layers[l];
    P.io = io;
    P.num_layers = num_layers;
    P.eps = dims.eps;
    P.inv_sqrt_d = 1.0f / sqrtf((float)D);
    const bool test_wait = (io.flags & GTM_DECODE_TEST_WAIT_RUNS_OUT) != 0;
    P.wait_limit_ns = test_wait ? 2000000ull : kTimeoutNs;
    P.first_wait_extra = test_wait ? 1u : 0u;
    unsigned char* w = static_cast<unsigned char*>(ws);
    P.logit_words = reinterpret_cast<unsigned long long*>(w);
    P.flags_b = reinterpret_cast<unsigned*>(w + 2048);
    P.flags_c = reinterpret_cast<unsigned*>(w + 3072);
    P.err = reinterpret_cast<int*>(w + kErrOffset);
    P.sticky = reinterpret_cast<int*>(w + kStickyOffset);
    float* f = reinterpret_cast<float*>(w + kDataOffset);
    P.act = f;
    P.part = P.act + FS + ACT_R;
    cudaError_t e = cudaMemsetAsync(w, 0, kErrOffset + sizeof(int), stream);
    if (e != cudaSuccess) return set_cuda_error("gtm_moe_decode: memset", e);
    const size_t smem = sizeof(Smem) + 128;
    static bool attr_done = false;
    if (!attr_done) {
        e = cudaFuncSetAttribute(moe_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return set_cuda_error("gtm_moe_decode: smem attribute", e);
        attr_done = true;
    }
    void* args[] = {(void*)&P};
    e = cudaLaunchCooperativeKernel((const void*)moe_decode_kernel, dim3(num_ctas), dim3(NT), args, smem, stream);
    if (e != cudaSuccess) return set_cuda_error("gtm_moe_decode: cooperative launch", e);
    return GTM_OK;
}

}  // namespace gtm
