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
// Per layer (one token), with bounded grid-wide waits:
//   tail    every CTA: layer tail of the previous layer from the down partials, optional
//           between-layer RMSNorm, views (dense_x, routed_x, router input), fragment tables
//   router  CTAs 0..127: their router logit in the reference's exact order (bit-identical), published
//           with the layer number in one 64-bit word; the words double as barrier A
//   shared  each CTA's share of the 264 shared gate/up tiles (+GeGLU)
//   top-8   wait for all 128 logit words; top-8 on every CTA; the producer starts the routed copies
//   routed  each CTA's share of the 704 routed gate/up tiles (+GeGLU)            -> barrier B
//   down    fragment tables of the 7744 activations; each CTA's share of the 1936 down items
//           (row tile x segment: 3 thirds of the shared down, 8 routed experts) -> barrier C
// The down partials [2 contributors][shared, routed][2816] are summed in fixed order by the tail.
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
constexpr int TILES_R = TOPK * FE / 8;    // 704 routed gate/up tiles (8 features each)
constexpr int TILES_S = FS / 8;           // 264 shared gate/up tiles
constexpr int TPE = FE / 8;               // 88 tiles per routed expert
constexpr int OT = D / 16;                // 176 output row tiles of the down projection
constexpr int NSEG = 3 + TOPK;            // down segments: 3 shared thirds + 8 routed experts
constexpr int ITEMS_DN = OT * NSEG;       // 1936 down items: row tile item / NSEG, segment item % NSEG
constexpr int ROW_GU = D / 2;             // 1408 bytes per gate/up row
constexpr int SROW_GU = GD * 2;           // 88 bytes of bf16 scales per gate/up row
constexpr int DROW_R = FE / 2, SROW_R = GFE * 2;   // routed down: 352 bytes per row, 22 of scales
constexpr int DROW_S = FS / 2, SROW_S = GFS * 2;   // shared down: 1056, 66
constexpr int RIN_PITCH = 65;
constexpr int QW = 192;                   // fragment-table words per quad: 2 double groups x 12 lane entries x 8
constexpr uint32_t RING = 144 * 1024;     // chunk ring
constexpr int NB = 32;                    // chunk mbarrier slots (> the chunks of any one phase)
constexpr int GU_TILES = 2;               // tiles per gate/up chunk
constexpr int MAX_DN = 24;                // down items per CTA (>= 1936 / 88)
constexpr int MAX_OTS = 4;                // down row tiles per CTA
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
    float* part;       // [2 contributors][2: shared, routed][D] down sums
};

// Per-CTA work lists (identical on every thread; derived from the CTA index and grid size).
struct Plan {
    int nr;              // router rows: cta, cta + G, ...
    int st0, st1;        // shared gate/up tiles
    int rt0, rt1;        // routed gate/up tiles
    int d0, d1;          // down items (row-tile-major)
    int n_sgu, n_rgu;    // gate/up chunks
    int ot0;             // first down row tile of the CTA
    int sh_a, sh_b;      // shared-down row tiles [sh_a, sh_b] of the shared-down chunk
    int c_sgu, c_rgu, c_dn, cpl;   // first chunk of each phase within a layer, chunks per layer
};

struct Smem {
    alignas(128) uint8_t ring[RING + 128];   // chunks (+ slack read by a down row's partial last quad)
    alignas(16) float hid[D];
    union {
        struct {
            alignas(16) float ab[2 * D];     // routed_x [0, D), dense_x [D, 2D)
            alignas(16) float rin[GD * RIN_PITCH];
        } t;
        alignas(16) uint32_t tbl_dn[NSEG * QS * QW];   // down inputs: segment q at q * 576 words
    } u;
    alignas(16) uint32_t tbl_r[QD * QW];     // routed_x
    alignas(16) uint32_t tbl_d[QD * QW];     // dense_x
    float2 gs_r[GD], gs_d[GD];               // per group of the views: (sum of x, 2^(E-6))
    float2 gs_dn[NSEG * 4 * QS];             // and of the down inputs
    float slot[SLOTS];                       // partial sums: [item][contributing warp k][16 rows]
    double red[2][NWC][2];
    float redf[2][NWC][2];
    double seq_sum;                          // certified RMS fallback
    float terms[GD];
    float topw[TOPK];
    int topi[TOPK];
    int dn_ot[MAX_DN], dn_q[MAX_DN];         // down items in processing (chunk) order
    uint8_t it_first[3][MAX_DN], it_kend[3][MAX_DN];   // per phase (shared, routed, down) and item:
                                                       // first contributing warp, contributors
    int dn_pos[MAX_OTS][NSEG];               // processing index of (row tile ot0 + i, segment q)
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
// Routed gate/up chunks: the CTA's tiles [rt0, rt1) cut at expert boundaries (every 88 tiles) and
// into pieces of at most GU_TILES.
__device__ __forceinline__ int rgu_next(const Plan& p, int s) {
    return min(min(p.rt1, (s / TPE + 1) * TPE), s + GU_TILES);
}
__device__ void rgu_chunk(const Plan& p, int k, int& t0, int& n) {
    int s = p.rt0;
    for (; k > 0; --k) s = rgu_next(p, s);
    t0 = s;
    n = rgu_next(p, s) - s;
}
__device__ void rgu_locate(const Plan& p, int T, int& k, int& t0) {
    int s = p.rt0;
    k = 0;
    for (;;) {
        const int e = rgu_next(p, s);
        if (T < e) { t0 = s; return; }
        s = e;
        ++k;
    }
}
// First / last down item of segment q in [d0, d1) (the range holds >= 11 items, so every segment).
__device__ __forceinline__ int seg_first(const Plan& p, int q) { return p.d0 + (q - p.d0 % NSEG + NSEG) % NSEG; }
__device__ __forceinline__ int seg_last(const Plan& p, int q) {
    return (p.d1 - 1) - ((p.d1 - 1) % NSEG - q + NSEG) % NSEG;
}

__device__ Plan make_plan(int cta, int G) {
    Plan p;
    p.nr = cta < NE ? (NE - 1 - cta) / G + 1 : 0;
    p.st0 = share(TILES_S, cta, G); p.st1 = share(TILES_S, cta + 1, G);
    p.rt0 = share(TILES_R, cta, G); p.rt1 = share(TILES_R, cta + 1, G);
    p.d0 = share(ITEMS_DN, cta, G); p.d1 = share(ITEMS_DN, cta + 1, G);
    p.n_sgu = (p.st1 - p.st0 + GU_TILES - 1) / GU_TILES;
    p.n_rgu = 0;
    for (int s = p.rt0; s < p.rt1; s = rgu_next(p, s)) ++p.n_rgu;
    p.ot0 = p.d0 / NSEG;
    p.sh_a = OT; p.sh_b = -1;
    for (int q = 0; q < 3; ++q) {
        p.sh_a = min(p.sh_a, seg_first(p, q) / NSEG);
        p.sh_b = max(p.sh_b, seg_last(p, q) / NSEG);
    }
    p.c_sgu = p.nr;
    p.c_rgu = p.c_sgu + p.n_sgu;
    p.c_dn = p.c_rgu + p.n_rgu;
    p.cpl = p.c_dn + 1 + TOPK;
    return p;
}

// Chunk i of a layer: ring bytes (copied; the allocation adds the 64-byte gate/up offset and rounds
// to 128) and whether it needs the layer's top-8.
__device__ uint32_t chunk_bytes(const Plan& p, int i) {
    if (i < p.c_sgu) return D;
    if (i < p.c_dn) {
        int nt;
        if (i < p.c_rgu) nt = min(GU_TILES, p.st1 - p.st0 - (i - p.c_sgu) * GU_TILES);
        else { int t0; rgu_chunk(p, i - p.c_rgu, t0, nt); }
        return (uint32_t)(8 * nt) * (2 * ROW_GU + 4 * SROW_GU);
    }
    if (i == p.c_dn) return (uint32_t)(16 * (p.sh_b - p.sh_a + 1)) * (DROW_S + 2 * SROW_S);
    const int q = 3 + (i - p.c_dn - 1);
    return (uint32_t)(16 * (seg_last(p, q) / NSEG - seg_first(p, q) / NSEG + 1)) * (DROW_R + 2 * SROW_R);
}

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
__device__ void l2_static(const Plan& p, const GtmLayer& L, const GtmLayer* Ln, int cta, int G) {
    const uint8_t* res = static_cast<const uint8_t*>(L.resident_dev);
    const uint32_t R = 16 * (p.sh_b - p.sh_a + 1), r0 = 16 * p.sh_a;
    tc::prefetch_l2_bulk(res + L.shared_down.weight + (uint64_t)r0 * DROW_S, R * DROW_S);
    tc::prefetch_l2_bulk(res + L.shared_down.scales + (uint64_t)r0 * SROW_S, R * SROW_S);
    tc::prefetch_l2_bulk(res + L.shared_down.biases + (uint64_t)r0 * SROW_S, R * SROW_S);
    if (!Ln) return;
    const uint8_t* rn = static_cast<const uint8_t*>(Ln->resident_dev);
    for (int k = 0; k < p.nr; ++k) tc::prefetch_l2_bulk(rn + Ln->router.weight + (uint64_t)(cta + k * G) * D, D);
    if (p.st1 > p.st0) {
        const uint64_t f0 = 8 * (uint64_t)p.st0, F = 8 * (uint64_t)(p.st1 - p.st0);
        tc::prefetch_l2_bulk(rn + Ln->shared_gate.weight + f0 * ROW_GU, F * ROW_GU);
        tc::prefetch_l2_bulk(rn + Ln->shared_up.weight + f0 * ROW_GU, F * ROW_GU);
        tc::prefetch_l2_bulk(rn + Ln->shared_gate.scales + f0 * SROW_GU, F * SROW_GU);
        tc::prefetch_l2_bulk(rn + Ln->shared_gate.biases + f0 * SROW_GU, F * SROW_GU);
        tc::prefetch_l2_bulk(rn + Ln->shared_up.scales + f0 * SROW_GU, F * SROW_GU);
        tc::prefetch_l2_bulk(rn + Ln->shared_up.biases + f0 * SROW_GU, F * SROW_GU);
    }
}

__device__ void producer(Smem& s, const Params& P, const Plan& p) {
    if ((threadIdx.x & 31) != 0) return;
    uint32_t head = 0, tail = 0;
    int issued = 0, released = 0;
    int tk[TOPK] = {0, 0, 0, 0, 0, 0, 0, 0};
    bool ok = true;
    const int cta = blockIdx.x, G = gridDim.x;
    for (int l = 0; l < P.num_layers && ok; ++l) {
        const GtmLayer& L = P.layers[l];
        const uint8_t* res = static_cast<const uint8_t*>(L.resident_dev);
        for (int i = 0; i < p.cpl && ok; ++i) {
            if (i == p.c_rgu) {   // the routed chunks follow: wait for this layer's top-8
                l2_static(p, L, l + 1 < P.num_layers ? &P.layers[l + 1] : nullptr, cta, G);
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
#pragma unroll
                for (int k = 0; k < TOPK; ++k) tk[k] = s.topi[k];
            }
            const uint32_t bytes = chunk_bytes(p, i);
            const uint32_t alloc = (bytes + 64 + 127) & ~127u;
            uint32_t pos = head % RING;
            if (pos + alloc > RING) { head += RING - pos; pos = 0; }
            while (head + alloc - tail > RING || issued - released >= NB) {
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
            if (i < p.c_sgu) {
                const int row = cta + i * G;
                tc::bulk_load(dst, res + L.router.weight + (uint64_t)row * D, D, bar);
            } else if (i < p.c_dn) {
                const bool routed = i >= p.c_rgu;
                int t0, nt;
                if (!routed) { t0 = p.st0 + (i - p.c_sgu) * GU_TILES; nt = min(GU_TILES, p.st1 - t0); }
                else rgu_chunk(p, i - p.c_rgu, t0, nt);
                const uint8_t* base = res;
                const GtmQuant *qg = &L.shared_gate, *qu = &L.shared_up;
                int f0 = 8 * t0;
                if (routed) {
                    base = rp(L.experts_dev, (uint64_t)tk[t0 / TPE] * L.expert_stride);
                    qg = &L.expert_gate;
                    qu = &L.expert_up;
                    f0 = 8 * (t0 % TPE);
                }
                const uint32_t F = 8 * nt, wb = F * ROW_GU, sb = F * SROW_GU;
                tc::bulk_load(dst, base + qg->weight + (uint64_t)f0 * ROW_GU, wb, bar);
                tc::bulk_load(dst + wb + 64, base + qu->weight + (uint64_t)f0 * ROW_GU, wb, bar);
                uint8_t* sd = dst + 2 * wb + 64;
                tc::bulk_load(sd, base + qg->scales + (uint64_t)f0 * SROW_GU, sb, bar);
                tc::bulk_load(sd + sb, base + qg->biases + (uint64_t)f0 * SROW_GU, sb, bar);
                tc::bulk_load(sd + 2 * sb, base + qu->scales + (uint64_t)f0 * SROW_GU, sb, bar);
                tc::bulk_load(sd + 3 * sb, base + qu->biases + (uint64_t)f0 * SROW_GU, sb, bar);
            } else if (i == p.c_dn) {
                const uint32_t R = 16 * (p.sh_b - p.sh_a + 1), r0 = 16 * p.sh_a;
                tc::bulk_load(dst, res + L.shared_down.weight + (uint64_t)r0 * DROW_S, R * DROW_S, bar);
                tc::bulk_load(dst + R * DROW_S, res + L.shared_down.scales + (uint64_t)r0 * SROW_S, R * SROW_S, bar);
                tc::bulk_load(dst + R * (DROW_S + SROW_S), res + L.shared_down.biases + (uint64_t)r0 * SROW_S,
                              R * SROW_S, bar);
            } else {
                const int q = 3 + (i - p.c_dn - 1);
                const int a = seg_first(p, q) / NSEG, b = seg_last(p, q) / NSEG;
                const uint32_t R = 16 * (b - a + 1), r0 = 16 * a;
                const uint8_t* blk = rp(L.experts_dev, (uint64_t)tk[q - 3] * L.expert_stride);
                tc::bulk_load(dst, blk + L.expert_down.weight + (uint64_t)r0 * DROW_R, R * DROW_R, bar);
                tc::bulk_load(dst + R * DROW_R, blk + L.expert_down.scales + (uint64_t)r0 * SROW_R, R * SROW_R, bar);
                tc::bulk_load(dst + R * (DROW_R + SROW_R), blk + L.expert_down.biases + (uint64_t)r0 * SROW_R,
                              R * SROW_R, bar);
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
// Tables of routed_x (ab[0, D)) and dense_x (ab[D, 2D)): 2 x 176 items, built by the compute
// threads from `first` on (whole warps: they take part in the builder's shuffles).
constexpr int VIEW_ITEMS = 2 * 4 * GD;
static_assert(VIEW_ITEMS % 32 == 0, "view-table items fill whole warps");
__device__ void build_views_tables(Smem& s, int first) {
    constexpr int N = VIEW_ITEMS;
    const int i0 = threadIdx.x - first;
    if (i0 < 0) return;
    if (i0 < ((N + 31) & ~31)) {
        const bool on = i0 < N;
        const int i = on ? i0 : (i0 & 3);
        const int v = i / (4 * GD), k = i - v * 4 * GD, j = k >> 2, sub = k & 3;
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

// Tables of the 11 down segments (act[704 q, 704 q + 704), written by every CTA before barrier B,
// read from L2): 11 x 12 groups x 4 items; group 11 of a segment (past its 704 inputs) is zero.
__device__ void build_down_tables(Smem& s, const Params& P) {
    constexpr int N = NSEG * 12 * 4;
    const int i0 = threadIdx.x;
    if (i0 < ((N + 31) & ~31)) {
        const bool on = i0 < N;
        const int i = on ? i0 : (i0 & 3);
        const int q = i / 48, k = i - q * 48, j = k >> 2, sub = k & 3;
        float x[16];
        if (j < GFE) {
            const float4* src = reinterpret_cast<const float4*>(P.act + q * FE + j * kGroup + 16 * sub);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float4 f = __ldcg(src + c);
                x[4 * c] = f.x; x[4 * c + 1] = f.y; x[4 * c + 2] = f.z; x[4 * c + 3] = f.w;
            }
        } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) x[e] = 0.0f;
        }
        limb_item(x, on, s.u.tbl_dn + q * QS * QW + (j >> 2) * QW, j & 3, sub, s.gs_dn + q * 12, j);
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

// Warp 0 polls every CTA's flag; the other compute warps wait at the named barrier.
__device__ bool wait_all(Smem& s, const Params& P, const unsigned* f, unsigned value) {
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        const uint64_t t0 = globaltimer_ns();
        bool ok = true;
        for (;;) {
            bool mine = true;
            for (unsigned b = lane; b < gridDim.x; b += 32) mine &= (ld_relaxed(f + b) >= value);
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
        // part [contributor][shared, routed][D]: shared = p00 + p10, routed h2 = p01 + p11
        const float4* pp = reinterpret_cast<const float4*>(P.part);
        const float4 p00 = __ldcg(pp + i), p01 = __ldcg(pp + D / 4 + i);
        const float4 p10 = __ldcg(pp + 2 * (D / 4) + i), p11 = __ldcg(pp + 3 * (D / 4) + i);
        float sh[4] = {p00.x + p10.x, p00.y + p10.y, p00.z + p10.z, p00.w + p10.w};
        float h2[4] = {p01.x + p11.x, p01.y + p11.y, p01.z + p11.z, p01.w + p11.w};
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
// Down items [d0, d1) in chunk order: the shared thirds (row tiles sh_a..sh_b, row-tile-major), then
// the 8 routed segments, each over its row tiles. dn_pos maps (row tile, segment) to that order.
__device__ void plan_down(Smem& s, const Plan& p) {
    if (threadIdx.x != 0) return;
    int k = 0;
    for (int it = p.d0; it < p.d1; ++it)
        if (it % NSEG < 3) { s.dn_ot[k] = it / NSEG; s.dn_q[k] = it % NSEG; ++k; }
    for (int q = 3; q < NSEG; ++q)
        for (int it = seg_first(p, q); it <= seg_last(p, q); it += NSEG) { s.dn_ot[k] = it / NSEG; s.dn_q[k] = q; ++k; }
    for (int a = 0; a < MAX_OTS; ++a)
        for (int q = 0; q < NSEG; ++q) s.dn_pos[a][q] = -1;
    for (int j = 0; j < k; ++j) s.dn_pos[s.dn_ot[j] - p.ot0][s.dn_q[j]] = j;
    fill_items(s, 0, p.st1 - p.st0, GD);
    fill_items(s, 1, p.rt1 - p.rt0, GD);
    fill_items(s, 2, p.d1 - p.d0, GFE);
}

__device__ bool down_phase(Smem& s, const Params& P, const Plan& p, int c_first) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const Split sp = make_split(p.d1 - p.d0, GFE);
    int pp = pw0(warp, sp.total);
    const int p1 = pw0(warp + 1, sp.total);
    int cur = c_first;
    bool ok = true;
    while (pp < p1) {
        const int k = pp / GFE, j0 = pp - k * GFE, j1 = min(GFE, j0 + (p1 - pp));
        const int ot = s.dn_ot[k], q = s.dn_q[k];
        const bool shared = q < 3;
        const int c = shared ? c_first : c_first + 1 + (q - 3);
        if (!advance_to(s, P, cur, c)) { ok = false; break; }
        const uint8_t* base = s.ring + s.meta[c % NB];
        const int first = shared ? p.sh_a : seg_first(p, q) / NSEG;
        const int last = shared ? p.sh_b : seg_last(p, q) / NSEG;
        const int R = 16 * (last - first + 1), row = 16 * (ot - first) + g;
        const int rowb = shared ? DROW_S : DROW_R, srow = shared ? GFS : GFE;   // bytes, scales per row
        const int kofs = shared ? q * GFE : 0;                                  // first group of the segment
        const uint8_t* w = base + (uint32_t)row * rowb + kofs * 32;
        const uint16_t* sc = reinterpret_cast<const uint16_t*>(base + (uint32_t)R * rowb) + row * srow + kofs;
        const uint16_t* bi = sc + R * srow;
        float ya = 0.0f, yb = 0.0f;
        tile_groups(w, w + 8 * rowb, sc, bi, sc + 8 * srow, bi + 8 * srow, j0, j1, s.u.tbl_dn + q * QS * QW,
                    s.gs_dn + q * 12, ya, yb);
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
    if (ok) ok = release_to(s, P, cur, c_first + 1 + TOPK);
    return ok;
}

// The CTA sums its segments of each row tile in segment order, shared and routed apart, into
// contributor slot 0 (the CTA holding segment 0 of the tile) or 1: a CTA holds >= 11 consecutive
// row-tile-major items, so a tile of 11 has at most two contributors, and the tail reads
// part[0] + part[1].
__device__ void down_epilogue(Smem& s, const Params& P, const Plan& p) {
    const Split sp = make_split(p.d1 - p.d0, GFE);
    const int ot1 = (p.d1 - 1) / NSEG;
    for (int i = threadIdx.x; i < (ot1 - p.ot0 + 1) * 16; i += NTC) {
        const int ot = p.ot0 + (i >> 4), r = i & 15;
        const int a = max(p.d0, ot * NSEG), b = min(p.d1, ot * NSEG + NSEG);
        float sh = 0.0f, h2 = 0.0f;
        for (int it = a; it < b; ++it) {
            const int q = it - ot * NSEG;
            const float v = item_sum(s, sp, 2, s.dn_pos[ot - p.ot0][q], r);
            if (q < 3) sh = __fadd_rn(sh, v);
            else h2 = __fadd_rn(h2, __fmul_rn(s.topw[q - 3], v));   // the product rounded, as the combine had it
        }
        const int c = a == ot * NSEG ? 0 : 1;
        float* pc = P.part + (size_t)c * 2 * D + ot * 16 + r;
        pc[0] = sh;
        pc[D] = h2;
        if (c == 0 && b == ot * NSEG + NSEG) {   // the whole tile here: no second contributor
            pc[2 * D] = 0.0f;
            pc[3 * D] = 0.0f;
        }
    }
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
    plan_down(s, p);
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

        // ---- router rows (the logit words double as barrier A) on warps 0-1, while warps 2-12
        //      build the fragment tables of the views ----
        int cur = cbase;
        bool ok = true;
        if (warp >= 2) build_views_tables(s, 64);
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
        csync();   // the view tables are complete

        // ---- shared gate/up ----
        if (ok && p.st1 > p.st0) {
            ok = gu_phase(s, P, 0, p.st1 - p.st0, cbase + p.c_sgu, cbase + p.c_rgu, s.tbl_d, s.gs_d,
                          [&](int item, int& c, int& lt, int& F) {
                              const int k = item / GU_TILES;
                              c = cbase + p.c_sgu + k;
                              lt = item - k * GU_TILES;
                              F = 8 * min(GU_TILES, p.st1 - p.st0 - k * GU_TILES);
                          });
            if (!ok) s.abort = 1;
            csync();
            if (!s.abort) gu_epilogue(s, 0, P.act + 8 * p.st0, p.st1 - p.st0);
        }
        csync();
        if (s.abort) break;

        // ---- wait for every router logit; top-8 ----
        if (warp == 0) {
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
        if (s.abort) break;

        // ---- routed gate/up ----
        ok = gu_phase(s, P, 1, p.rt1 - p.rt0, cbase + p.c_rgu, cbase + p.c_dn, s.tbl_r, s.gs_r,
                      [&](int item, int& c, int& lt, int& F) {
                          int k, t0;
                          rgu_locate(p, p.rt0 + item, k, t0);
                          int tt, nt;
                          rgu_chunk(p, k, tt, nt);
                          c = cbase + p.c_rgu + k;
                          lt = p.rt0 + item - t0;
                          F = 8 * nt;
                      });
        if (!ok) s.abort = 1;
        csync();
        if (s.abort) break;
        gu_epilogue(s, 1, P.act + FS + 8 * p.rt0, p.rt1 - p.rt0);
        arrive(P, P.flags_b, ep);

        // ---- down: the shared and routed activations of every CTA ----
        if (!wait_all(s, P, P.flags_b, ep)) break;
        build_down_tables(s, P);
        csync();
        ok = down_phase(s, P, p, cbase + p.c_dn);
        if (!ok) s.abort = 1;
        csync();
        if (s.abort) break;
        down_epilogue(s, P, p);
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
    return kDataOffset + sizeof(float) * (dec::ACT_R + dec::FS + (size_t)4 * dec::D) + 256;
}
size_t decode_sticky_offset() { return kStickyOffset; }

int launch_decode(const GtmDims& dims, const GtmLayer* layers, int num_layers, const GtmDecodeIO& io,
                  void* ws, size_t ws_bytes, cudaStream_t stream, int num_ctas) {
    using namespace dec;
    (void)ws_bytes;
    if (num_ctas > OT || num_ctas * MAX_DN < ITEMS_DN)
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
