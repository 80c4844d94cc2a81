// grouped_tc.cu — block-scaled tensor-core (tcgen05 / TMEM) grouped pass for MX weights.
//
// The weights never leave their MX encoding: a 128-row x 128-byte tile (E2M1 nibbles or E4M3
// bytes, pre-swizzled for the 128-byte canonical K-major layout, followed by its E8M0 scales in
// the tcgen05.cp chunk layout) is one contiguous run of HBM that one 1-D bulk copy (TMA engine)
// drops into shared memory, where tcgen05.mma kind::mxf4 / kind::mxf8f6f4 reads it directly.
// No CUDA-core dequantisation remains on the weight stream, so the pass runs at the rate HBM
// delivers tiles.
//
// BF16 weights (kind::f16) are not repacked: each 128-row x 64-column tile is a 2-D tiled TMA
// copy from the row-major matrix through its tensor map, landing in the same 128-byte swizzled
// K-major layout; they carry no scales.
//
// Activations are represented in the weights' element format by residual terms (k_bs_prep):
// per 32-column block, term j takes the E8M0 scale that fits the residual's largest magnitude
// into the element range (6 for E2M1, 448 for E4M3), rounds to nearest, and passes the
// remainder to term j+1.  Each token owns bs_rows_per_tok consecutive MMA rows (its terms, then
// zero rows); the epilogue adds the term columns of a token.
//
// One persistent CTA per SM walks work units (group, 128-row tile, sub-segment).  tcgen05
// instructions cost ~120-200 cycles of issue each on the issuing thread, while MMAs issued from
// several threads proceed concurrently, so the per-stage instruction stream is spread over
// warps:
//   warp 0 (one thread)  weight producer: tiles into an 8-slot ring (bulk copies, mbarriers);
//   warp 3 (one thread)  activation producer: stages into a byte ring (variable-size stages,
//                        up to 16 in flight) from their L2-resident source;
//   warps 8-11           scale warps: each stage's E8M0 scales of both operands from shared
//                        memory into TMEM with tcgen05.st (each warp fills its lane quarter);
//   warps 1, 2           MMA issuers (one thread each), each into its own TMEM accumulator;
//   warps 4-7, 12-15     epilogue: tcgen05.ld of the accumulators, term sums, results out
//                        (the accumulator is released before the results are stored).
// Down pass: a group is one matrix; the issuers split each stage's 4 K steps, release stages
// two at a time (one tcgen05.commit on the pair's barrier, a 32-deep ring both producers
// watch), and the epilogue adds their halves and stores f32 output rows.
// Gate/up pass (paired groups): a stage brings the gate tile and the up tile of one expert
// (two ring slots) against one activation stage; issuer 0 runs the gate MMAs, issuer 1 the up
// MMAs (all four K steps each), every stage is released on its own barrier, and the epilogue
// forms h = silu(gate) * up and writes it as f32 rows (one per column), the down pass's prep
// source.
// Units of N <= 64 MMA rows alternate between two 64-column halves of the accumulators, so the
// epilogue of one unit overlaps the MMAs of the next.
#include "bs_terms.cuh"
#include "numerics.cuh"
#include "tc_common.cuh"
#include "urb_internal.cuh"
#include "urb_tc.cuh"

namespace urb {
namespace {

constexpr int kSA = 8;                // weight ring depth (also the TMEM scale slots)
constexpr int kStage = 17408;         // bytes of one weight slot / largest activation stage
constexpr int kBRing = 5 * kStage;    // activation byte ring
constexpr int kSB = 16;               // activation stages in flight at most
constexpr int kRel = 32;              // release barriers, one per pair of stages (covers 64)
constexpr int kIssuers = kBsIssuers;
constexpr int kStepsPerIssuer = 4 / kIssuers;
static_assert(kIssuers == 2, "issuers");
// Warps: 0 weight producer, 1-2 issuers, 3 activation producer, 4-7 and 12-15 epilogue, 8-11
// scale warps.  Each polling thread sits on its own scheduler (warp % 4).
constexpr int kThreadsBs = 512;
constexpr int kWarpBProd = 3;
constexpr uint32_t kAccCols = kBsNmax;  // accumulator columns per issuer
constexpr uint32_t kSfCol0 = kIssuers * kAccCols;  // first scale column: slot s at +16 s
constexpr int kSmemBs = kSA * kStage + kBRing + 1024;

static_assert(bs_tile_bytes(URB_FMT_MXFP4) <= kStage && bs_tile_bytes(URB_FMT_MXFP8) <= kStage, "slot");
static_assert(bs_bstage_bytes(URB_FMT_MXFP4, kBsNmax) <= kStage, "slot");
static_assert(kSfCol0 + kSA * 16 <= 512, "tmem");
static_assert(kAccCols % 32 == 0, "accumulator alignment");
static_assert(2 * kRel >= kSA + kSB + 2, "release-barrier ring too short");
static_assert(kSmemBs <= 227 * 1024 - 1024, "shared memory");

__device__ __forceinline__ void set_status(int32_t *status, int code) {
    if (status) atomicCAS(status, 0, int32_t(code));
}

// Walks the work units of this CTA (u = blockIdx.x, += gridDim.x).  The group of the next
// unit is loaded one unit ahead and its group index two units ahead, so a role never waits on
// a global load at a unit boundary.
struct UnitCursor {
    const TcSeg *segs;
    const int *map;
    int u, step, total;
    TcSeg cur, nxt;
    int g2;
    __device__ __forceinline__ UnitCursor(const TcArgs &a, int total_units)
        : segs(a.segs), map(a.unit_group), u(blockIdx.x), step(gridDim.x), total(total_units) {
        if (u < total) cur = segs[map[u]];
        if (u + step < total) nxt = segs[map[u + step]];
        g2 = u + 2 * step < total ? map[u + 2 * step] : 0;
    }
    __device__ __forceinline__ bool valid() const { return u < total; }
    __device__ __forceinline__ void advance() {
        u += step;
        cur = nxt;
        if (u + step < total) nxt = segs[g2];
        if (u + 2 * step < total) g2 = map[u + 2 * step];
    }
};

__device__ __forceinline__ int round16i(int v) { return (v + 15) & ~15; }

// Stage p has been consumed once its pair's release barrier has fired (the issuers commit after
// every odd stage and after the last stage of the launch).
// Paired groups (two weight tiles per stage) release every stage on its own barrier.
template <bool PAIR>
__device__ __forceinline__ bool wait_consumed(uint64_t *rel, uint32_t p, volatile int *abort) {
    const uint32_t r = PAIR ? p : p >> 1;
    return tc::mbar_wait(&rel[r % kRel], (r / kRel) & 1, abort);
}

struct Unit {
    int mt, sub, nt, n;
};

// Accumulator halves.  A unit of N <= 64 MMA rows takes one 64-column half of each issuer's
// accumulator, alternating, so the epilogue drains one unit while the issuers fill the other
// half with the next; a wider unit takes both halves.  Issuers and epilogue walk the same
// units, so both derive the same assignment.
struct AccHalves {
    uint32_t next = 0;           // half for the next narrow unit
    uint32_t use[2] = {0, 0};    // units that have used each half so far
    uint32_t full[2] = {0, 0};   // completions of each half's full barrier seen so far
    __device__ __forceinline__ uint32_t mask_of(int n) {  // halves used by a unit of N rows
        if (n <= 64) {
            const uint32_t h = next;
            next ^= 1u;
            return 1u << h;
        }
        next = 0;
        return 3u;
    }
};
__device__ __forceinline__ uint32_t first_half(uint32_t mask) { return mask == 2u ? 1u : 0u; }
// TPU: row tiles per unit (2 when neighbouring tiles are paired).
template <int FMT, int TPU = 1>
__device__ __forceinline__ Unit unit_of(const TcSeg &S, int u) {
    Unit x;
    const int r = u - S.unit_begin;
    const int mu = r / S.nsub;
    x.sub = r - mu * S.nsub;
    x.mt = mu * TPU;
    x.nt = min(bs_cap(FMT), S.ntok - x.sub * bs_cap(FMT));
    x.n = round16i(bs_rows_per_tok(FMT) * x.nt);
    return x;
}

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }
// The gate/up epilogue's silu on the f32 path: the hardware exp2 and reciprocal (a few
// instructions instead of the accurate expf and the IEEE division, whose range checks and slow
// path dominated the epilogue).  Relative error below 2e-5 for |v| < 88 (__expf's error grows
// with |v|); beyond, 1 + e^-v is infinite and the result is -0, as in the IEEE form.
__device__ __forceinline__ float silu_fast(float v) { return __fdividef(v, 1.0f + __expf(-v)); }

// MODE 1 (gate/up pass): each group carries the gate (w) and up (w2) tiles of one expert; a
// stage brings both tiles and one activation stage, issuer 0 runs the gate MMAs and issuer 1 the
// up MMAs (all four K steps each), and the epilogue writes h = silu(gate) * up.
// MODE 2 (down pass, paired row tiles): a unit covers row tiles mt and mt + 1 of one matrix;
// a stage brings both tiles against one activation stage, issuer i runs tile mt + i (all four
// K steps), and the epilogue writes both tiles' output rows (a missing last tile of an odd
// count is neither copied nor multiplied).
// MODE 0: the issuers split each stage's K steps of one tile; the epilogue adds their halves.
template <int FMT, int MODE, int NT>
__global__ void __launch_bounds__(kThreadsBs, 1) k_bs_grouped(TcArgs a) {
    grid_dep_wait();  // programmatic dependent launch: the kernel ahead has completed
    grid_dep_trigger();
    constexpr bool PAIR = MODE != 0;   // two weight tiles per stage, one per issuer
    constexpr bool GU = MODE == 1, MT = MODE == 2;
    constexpr int TPU = MT ? 2 : 1;    // row tiles per unit
    static_assert(!PAIR || kIssuers == 2, "paired tiles run one issuer per tile");
    constexpr int TPS = PAIR ? 2 : 1;  // weight tiles per stage
    // Weight slots and activation ring bytes.  The copies of a stage are bound by the SM's
    // intake (~55 B per cycle from L2 for re-read tiles), so the copy latency grows with the ring
    // depth; 8 weight slots / 5 activation stages measured 3-6 % faster than 6 / 7 on config 2,
    // on config 3 and on 32 tokens per expert (10 / 3 starves the activation ring).
    constexpr int SA = kSA;
    constexpr int BRING = kBRing;
    constexpr int TB = bs_tile_bytes(FMT);
    constexpr int CH = bs_sf_chunks(FMT);
    constexpr int KIND_FMT = FMT == URB_FMT_MXFP4 ? 1 : 0;
    constexpr bool BF = FMT == URB_FMT_BF16;  // kind::f16, tiles through the tensor map, no scales
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *ring_a = smem;
    uint8_t *ring_b = smem + size_t(SA) * kStage;
    __shared__ __align__(8) uint64_t a_full[SA], sf_full[SA], b_full[kSB], rel[kRel];
    __shared__ __align__(8) uint64_t acc_full[2], acc_empty[2], mma_done[kIssuers];
    __shared__ uint32_t b_off[kSB];  // byte offset of each in-flight activation stage
    __shared__ uint32_t tmem_base;
    __shared__ int abort_flag, skip, never;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nsegs = *a.nsegs;
    const int total_units = *a.total_units;
    if (threadIdx.x == 0) skip = (total_units <= 0 || nsegs <= 0 || (a.status && *a.status)) ? 1 : 0;
    __syncthreads();
    if (skip) return;

    if (threadIdx.x == 0) {
        for (int s = 0; s < SA; ++s) {
            tc::mbar_init(&a_full[s], 1);
            tc::mbar_init(&sf_full[s], 4);   // one arrival per scale warp
        }
        for (int s = 0; s < kSB; ++s) tc::mbar_init(&b_full[s], 1);
        for (int s = 0; s < kRel; ++s) tc::mbar_init(&rel[s], kIssuers);  // one commit per issuer
        for (int h = 0; h < 2; ++h) {
            tc::mbar_init(&acc_full[h], kIssuers);
            tc::mbar_init(&acc_empty[h], 8);  // one arrival per epilogue warp
        }
        for (int s = 0; s < kIssuers; ++s) tc::mbar_init(&mma_done[s], 1);
        tc::mbar_fence_init();
        abort_flag = 0;
        never = 0;
    }
    if (warp == 1) {
        tc::tmem_alloc(&tmem_base, 512);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tbase = tmem_base;
    volatile int *abortp = &abort_flag;
    auto fail = [&]() {
        *abortp = 1;
        set_status(a.status, URB_ERR_TIMEOUT);
    };

    if (warp == 0 && lane == 0) {
        // ---------------- weight producer ----------------
        uint32_t g = 0;  // tiles issued (stage * TPS + i)
        for (UnitCursor uc(a, total_units); uc.valid() && !*abortp; uc.advance()) {
            const TcSeg &S = uc.cur;
            const Unit x = unit_of<FMT, TPU>(S, uc.u);
            // MX: tile (mt, ks) at (ks * mts + mt) of the resident tiles.  BF16: box (column
            // 64 ks, row 128 mt) of the tensor map (S.w / S.w2 point at the maps).
            const uint8_t *wsrc = BF ? S.w : S.w + size_t(x.mt) * TB;
            const uint8_t *wsrc2 = GU ? (BF ? S.w2 : S.w2 + size_t(x.mt) * TB)
                                      : (MT ? (BF ? S.w : S.w + size_t(x.mt + 1) * TB) : nullptr);
            const bool second = !MT || x.mt + 1 < S.mts;  // the unit's second tile exists
            bool ok = true;
            for (int ks = 0; ks < S.ks && ok; ++ks) {
#pragma unroll
                for (int i = 0; i < TPS; ++i, ++g) {
                    const int sa = int(g % SA);
                    // The slot is free once the stage of the tile it held has been consumed.
                    if (g >= uint32_t(SA) && !wait_consumed<PAIR>(rel, (g - SA) / TPS, abortp)) {
                        ok = false;
                        break;
                    }
                    if (i == 1 && !second) {  // no tile: complete the slot's phase empty
                        tc::mbar_arrive(&a_full[sa]);
                        continue;
                    }
                    tc::mbar_arrive_expect_tx(&a_full[sa], uint32_t(TB));
                    if constexpr (BF)
                        tc::tma_load_2d(ring_a + size_t(sa) * kStage, i ? wsrc2 : wsrc,
                                        ks * bs_stage_cols(FMT), (x.mt + (MT ? i : 0)) * 128, &a_full[sa]);
                    else
                        tc::bulk_g2s(ring_a + size_t(sa) * kStage,
                                     (i ? wsrc2 : wsrc) + size_t(ks) * S.mts * TB, TB, &a_full[sa]);
                }
            }
            if (!ok) { fail(); break; }
        }
        // Let every copy this thread issued land before the CTA can exit.
        for (uint32_t i = g > uint32_t(SA) ? g - SA : 0; i < g; ++i)
            tc::mbar_wait(&a_full[i % SA], (i / SA) & 1, &never);
    } else if (warp == kWarpBProd && lane == 0) {
        // ---------------- activation producer ----------------
        // Byte ring: stage g occupies [q_start, q_end) (1 KB granules, contiguous) until stage g
        // has been consumed; the oldest in-flight stage is retired by waiting on its release
        // barrier.  At most kSB stages are in flight.
        uint32_t q_start[kSB];
        uint32_t g = 0, oldest = 0, head = 0;
        for (UnitCursor uc(a, total_units); uc.valid() && !*abortp; uc.advance()) {
            const TcSeg &S = uc.cur;
            const Unit x = unit_of<FMT, TPU>(S, uc.u);
            const uint32_t bbytes = uint32_t(bs_bstage_bytes(FMT, x.n));
            const uint32_t need = (bbytes + 1023) & ~1023u;
            const uint8_t *bsrc = a.bbuf + S.b_off + (long long)x.sub * S.ks * bs_bstage_bytes(FMT, kBsNmax);
            bool ok = true;
            for (int ks = 0; ks < S.ks && ok; ++ks, ++g) {
                uint32_t pos = 0;
                for (;;) {
                    const uint32_t inflight = g - oldest;
                    if (inflight == 0) { head = 0; pos = 0; break; }
                    if (inflight < uint32_t(kSB)) {
                        const uint32_t tail = q_start[oldest % kSB];
                        // Both wrapped placements are strict: a wrapped ring never fills up to
                        // its tail, so head == tail only ever means "nothing in flight".
                        if (head >= tail) {  // used [tail, head): free [head, end) and [0, tail)
                            if (head + need <= uint32_t(BRING)) { pos = head; break; }
                            if (need < tail) { pos = 0; break; }
                        } else if (head + need < tail) {  // used [tail, end) + [0, head)
                            pos = head;
                            break;
                        }
                    }
                    if (!wait_consumed<PAIR>(rel, oldest, abortp)) { ok = false; break; }
                    ++oldest;
                }
                if (!ok) break;
                const int sb = int(g % kSB);
                q_start[sb] = pos;
                head = pos + need;
                b_off[sb] = pos;
                tc::mbar_arrive_expect_tx(&b_full[sb], bbytes);
                tc::bulk_g2s(ring_b + pos, bsrc + size_t(ks) * bbytes, bbytes, &b_full[sb]);
            }
            if (!ok) { fail(); break; }
        }
        for (uint32_t i = g > uint32_t(kSB) ? g - kSB : 0; i < g; ++i)
            tc::mbar_wait(&b_full[i % kSB], (i / kSB) & 1, &never);
    } else if (warp >= 8 && warp < 12) {
        // ---------------- scale warps ----------------
        // TMEM scale slot sa (16 columns): A's chunks at +0 / +4, B's at +8 / +12; lane l of
        // every quarter holds bytes 16 l .. 16 l + 15 of each 512-byte chunk.
        const uint32_t lane_base = uint32_t(32 * (warp & 3)) << 16;
        uint32_t g = 0;
        for (UnitCursor uc(a, total_units); uc.valid() && !*abortp; uc.advance()) {
            const TcSeg &S = uc.cur;
            const Unit x = unit_of<FMT, TPU>(S, uc.u);
            bool ok = true;
            for (int ks = 0; ks < S.ks; ++ks, ++g) {
                const uint32_t t0 = g * TPS;  // first weight tile of the stage
                const int sa = int(t0 % SA), sa1 = int((t0 + TPS - 1) % SA), sb = int(g % kSB);
                if (!tc::mbar_wait(&a_full[sa], (t0 / SA) & 1, abortp) ||
                    (PAIR && !tc::mbar_wait(&a_full[sa1], ((t0 + 1) / SA) & 1, abortp)) ||
                    !tc::mbar_wait(&b_full[sb], (g / kSB) & 1, abortp)) {
                    ok = false;
                    break;
                }
                if constexpr (BF) {  // no scales: only tell the issuers that the stage landed
                    __syncwarp();
                    if (lane == 0) tc::mbar_arrive(&sf_full[sa]);
                    continue;
                }
                // Slot sa: A's scales at +0 / +4, B's at +8 / +12; PAIR: the up tile's A scales
                // in its own slot sa1 (+0 / +4).
                const uint8_t *sfa = ring_a + size_t(sa) * kStage + 16384 + 16 * lane;
                const uint8_t *sfa1 = ring_a + size_t(sa1) * kStage + 16384 + 16 * lane;
                const uint8_t *sfb = ring_b + b_off[sb] + x.n * 128 + 16 * lane;
                uint32_t v[16], v1[16];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    uint4 qa = make_uint4(0, 0, 0, 0), qb = make_uint4(0, 0, 0, 0);
                    uint4 qa1 = make_uint4(0, 0, 0, 0);
                    if (h < CH) {
                        qa = *reinterpret_cast<const uint4 *>(sfa + 512 * h);
                        qb = *reinterpret_cast<const uint4 *>(sfb + 512 * h);
                        if (PAIR) qa1 = *reinterpret_cast<const uint4 *>(sfa1 + 512 * h);
                    }
                    v[4 * h] = qa.x; v[4 * h + 1] = qa.y; v[4 * h + 2] = qa.z; v[4 * h + 3] = qa.w;
                    v[8 + 4 * h] = qb.x; v[9 + 4 * h] = qb.y; v[10 + 4 * h] = qb.z; v[11 + 4 * h] = qb.w;
                    v1[4 * h] = qa1.x; v1[4 * h + 1] = qa1.y; v1[4 * h + 2] = qa1.z; v1[4 * h + 3] = qa1.w;
                    v1[8 + 4 * h] = 0; v1[9 + 4 * h] = 0; v1[10 + 4 * h] = 0; v1[11 + 4 * h] = 0;
                }
                tc::tmem_st16(tbase + lane_base + kSfCol0 + 16u * sa, v);
                if (PAIR) tc::tmem_st16(tbase + lane_base + kSfCol0 + 16u * sa1, v1);
                tc::wait_st();
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&sf_full[sa]);
            }
            if (!ok) { fail(); break; }
        }
    } else if ((warp == 1 || warp == 2) && lane == 0) {
        // ---------------- MMA issuers (their K steps of every stage) ----------------
        const int me = warp - 1;
        uint32_t g = 0;
        AccHalves ah;
        for (UnitCursor uc(a, total_units); uc.valid() && !*abortp; uc.advance()) {
            const TcSeg &S = uc.cur;
            const Unit x = unit_of<FMT, TPU>(S, uc.u);
            const uint32_t mask = ah.mask_of(x.n), h0 = first_half(mask);
            const uint32_t acc = tbase + uint32_t(me) * kAccCols + 64u * h0;
            bool empty_ok = true;
            for (uint32_t h = 0; h < 2; ++h) {
                if (!(mask >> h & 1u)) continue;
                if (ah.use[h] >= 1 && !tc::mbar_wait(&acc_empty[h], (ah.use[h] - 1) & 1, abortp))
                    empty_ok = false;
                ++ah.use[h];
            }
            if (!empty_ok) { fail(); break; }
            tc::fence_after_sync();
            bool ok = true;
            for (int ks = 0; ks < S.ks; ++ks, ++g) {
                const uint32_t t0 = g * TPS;
                const int sa = int(t0 % SA), sb = int(g % kSB);
                // PAIR: issuer i multiplies the stage's tile i (gate / up, or row tile mt + i).
                const int sam = PAIR ? int((t0 + uint32_t(me)) % SA) : sa;
                const bool idle = MT && me == 1 && x.mt + 1 >= S.mts;  // no second tile
                // The scale warps arrive only after every copy of the stage has landed.
                if (!tc::mbar_wait(&sf_full[sa], (t0 / SA) & 1, abortp)) { ok = false; break; }
                tc::fence_after_sync();
                const uint32_t sA = tc::smem_u32(ring_a + size_t(sam) * kStage);
                const uint32_t sB = tc::smem_u32(ring_b + b_off[sb]);
                const uint32_t sfa = tbase + kSfCol0 + 16u * sam, sfb = tbase + kSfCol0 + 16u * sa + 8;
                const uint64_t adesc = tc::sdesc_sw128(sA), bdesc = tc::sdesc_sw128(sB);
                constexpr int kSteps = PAIR ? 4 : kStepsPerIssuer;
#pragma unroll
                for (int k2 = 0; k2 < kSteps && !idle; ++k2) {
                    const int kk = PAIR ? k2 : me * kStepsPerIssuer + k2;
                    const bool accum = ks > 0 || k2 > 0;
                    if constexpr (BF) {
                        tc::mma_bf16(acc, adesc + 2 * kk, bdesc + 2 * kk, tc::idesc_bf16(x.n), accum);
                    } else if (FMT == URB_FMT_MXFP4) {
                        const uint32_t id = 2u * (kk & 1), col = 4u * (kk >> 1);
                        tc::mma_mxf4(acc, adesc + 2 * kk, bdesc + 2 * kk, tc::idesc_bs(KIND_FMT, x.n, id, id),
                                     (sfa + col) | (id << 30), (sfb + col) | (id << 30), accum);
                    } else {
                        const uint32_t id = uint32_t(kk);
                        tc::mma_mxf8(acc, adesc + 2 * kk, bdesc + 2 * kk, tc::idesc_bs(KIND_FMT, x.n, id, id),
                                     sfa | (id << 30), sfb | (id << 30), accum);
                    }
                }
                const bool last = ks == S.ks - 1 && uc.u + uc.step >= uc.total;
                if (PAIR) tc::mma_commit(&rel[g % kRel]);
                else if ((g & 1) || last) tc::mma_commit(&rel[(g >> 1) % kRel]);
                if (ks == S.ks - 1) tc::mma_commit(&acc_full[h0]);
            }
            if (!ok) { fail(); break; }
        }
        // Every MMA of this thread completes before TMEM is released.
        tc::mma_commit(&mma_done[me]);
        tc::mbar_wait(&mma_done[me], 0, &never);
    } else if ((warp >= 4 && warp < 8) || warp >= 12) {
        // ---------------- epilogue ----------------
        // Two groups of four warps (4-7, 12-15), one warp per TMEM lane quarter in each, take
        // the even / odd 16-column chunks of a unit.  A warp reads its chunks, forms its
        // results in registers and releases the accumulator before it stores anything, so the
        // issuers wait only for the TMEM reads at a unit boundary.
        constexpr int RT = bs_rows_per_tok(FMT), TT = NT, TPC = 16 / RT;
        constexpr int MYCH = kBsNmax / 32;  // chunks of a full-width unit per group
        constexpr int NOUT = MT ? 2 : 1;    // outputs per (row, token): the down pass's two tiles
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        const int eg = warp >= 12 ? 1 : 0;
        const int row = 32 * q + lane;
        const uint32_t lane_base = uint32_t(32 * q) << 16;
        AccHalves ah;
        for (UnitCursor uc(a, total_units); uc.valid() && !*abortp; uc.advance()) {
            const TcSeg &S = uc.cur;
            const Unit x = unit_of<FMT, TPU>(S, uc.u);
            const uint32_t mask = ah.mask_of(x.n), h0 = first_half(mask);
            if (!tc::mbar_wait(&acc_full[h0], ah.full[h0]++ & 1, abortp)) { fail(); break; }
            tc::fence_after_sync();
            const int grow = x.mt * 128 + row;
            const bool row_ok = grow < S.rows;
            const int tok0 = x.sub * bs_cap(FMT);
            const int nch = x.n / 16;
            float res[MYCH][TPC][NOUT];
#pragma unroll
            for (int j = 0; j < MYCH; ++j) {
                const int c = 2 * j + eg;
                if (c >= nch) break;  // uniform across the warp
                uint32_t v[kIssuers][16];
#pragma unroll
                for (int i = 0; i < kIssuers; ++i)
                    tc::tmem_ld16(tbase + lane_base + uint32_t(i) * kAccCols + 64u * h0 + 16 * c, v[i]);
                tc::wait_ld();
#pragma unroll
                for (int s = 0; s < TPC; ++s) {
                    const int t = TPC * c + s;
                    if (t >= x.nt) continue;
                    if constexpr (MT) {
                        // Accumulator i holds row tile mt + i.
#pragma unroll
                        for (int i = 0; i < 2; ++i) {
                            float o = 0.0f;
#pragma unroll
                            for (int e = 0; e < TT; ++e) o += __uint_as_float(v[i][RT * s + e]);
                            if (a.variant != 0) o = num_round_bf16(o);
                            if (a.variant == 2 && !isfinite(o) && x.mt + i < S.mts &&
                                (x.mt + i) * 128 + row < S.rows)
                                set_status(a.status, URB_ERR_NONFINITE);
                            res[j][s][i] = o;
                        }
                    } else if constexpr (GU) {
                        // h = silu(gate) * up of this lane's row.
                        float gv = 0.0f, uv = 0.0f;
#pragma unroll
                        for (int e = 0; e < TT; ++e) {
                            gv += __uint_as_float(v[0][RT * s + e]);
                            uv += __uint_as_float(v[1][RT * s + e]);
                        }
                        float h;
                        if (a.variant == 1) {
                            h = num_bounded_swiglu(num_round_bf16(gv), num_round_bf16(uv), a.limit);
                            h = num_round_bf16(__fmul_rn(h, a.col_w[S.col_begin + tok0 + t]));
                        } else if (a.variant == 2) {
                            const float act = num_round_bf16(num_silu_libm(num_round_bf16(gv), a.expf));
                            h = num_round_bf16(__fmul_rn(act, num_round_bf16(uv)));
                        } else {
                            h = silu_fast(gv) * uv;
                        }
                        if (a.variant != 0 && row_ok && !isfinite(h)) set_status(a.status, URB_ERR_NONFINITE);
                        res[j][s][0] = h;
                    } else {
                        float o = 0.0f;
#pragma unroll
                        for (int e = 0; e < TT; ++e)
                            o += __uint_as_float(v[0][RT * s + e]) + __uint_as_float(v[1][RT * s + e]);
                        if (a.variant != 0) o = num_round_bf16(o);
                        if (a.variant == 2 && row_ok && !isfinite(o)) set_status(a.status, URB_ERR_NONFINITE);
                        res[j][s][0] = o;
                    }
                }
            }
            // Every TMEM read of this warp has completed: the issuers may overwrite the halves.
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0)
                for (uint32_t h = 0; h < 2; ++h)
                    if (mask >> h & 1u) tc::mbar_arrive(&acc_empty[h]);
#pragma unroll
            for (int j = 0; j < MYCH; ++j) {
                const int c = 2 * j + eg;
                if (c >= nch) break;
#pragma unroll
                for (int s = 0; s < TPC; ++s) {
                    const int t = TPC * c + s;
                    if (t >= x.nt) continue;
                    const int col = S.col_begin + tok0 + t;
                    if constexpr (GU) {
                        if (row_ok) a.out[size_t(col) * a.out_stride + grow] = res[j][s][0];
                        continue;
                    }
                    float *dst;
                    if (a.out_ranks && col < a.routed_cols) {
                        const int i = a.out_rows[col];
                        dst = a.out_ranks[i / a.out_rank_rows] + size_t(i % a.out_rank_rows) * a.out_stride;
                    } else {
                        dst = a.out + size_t(a.out_ranks ? col - a.routed_cols : col) * a.out_stride;
                    }
#pragma unroll
                    for (int i = 0; i < NOUT; ++i) {
                        const int gr = (x.mt + i) * 128 + row;
                        if (x.mt + i >= S.mts || gr >= S.rows) continue;
                        dst[S.out_off + gr] = res[j][s][i];
                    }
                }
            }
        }
        // Rows stored into other ranks' memory are visible system-wide before the exchange
        // barrier that follows this launch signals them.
        if (a.out_ranks) __threadfence_system();
    }
    // Every lane of a role warp waits for its lane 0 here, so the CTA barrier below is reached
    // by converged warps only.
    __syncwarp();
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tbase, 512);
    }
}

// Activation stages.  A lane quad per (source row, 32-column block), 8 columns per lane:
// loads the block (x, or h = silu(gate) * up), builds the residual terms once and writes them
// into every activation column that uses the row (gate/up: the token's routed positions and
// the shared expert's column), as MMA rows slot * rows_per_tok + term of the column's
// sub-segment (payload 128-byte swizzled, scale bytes in the tcgen05.cp chunk layout).  MMA rows
// past a token's terms and slots past a sub-segment's tokens are never read by the epilogue
// and stay unwritten.
// BF16 (round to nearest even) of a finite f32, as the 16 high bits of its pattern.
__device__ __forceinline__ uint32_t bf16_bits_rn(float v) {
    const uint32_t u = __float_as_uint(v);
    return (u + 0x7FFFu + ((u >> 16) & 1u)) >> 16;
}

// One BF16 residual term of a lane's 8 values: q receives the 8 BF16 codes (element 0 in the
// low half of word 0) and r the exact remainder.  Three terms reproduce an f32 exactly.
__device__ __forceinline__ void make_term8_bf16(float *r, uint32_t *q) {
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
        const uint32_t b0 = bf16_bits_rn(r[i]), b1 = bf16_bits_rn(r[i + 1]);
        r[i] -= __uint_as_float(b0 << 16);
        r[i + 1] -= __uint_as_float(b1 << 16);
        q[i >> 1] = b0 | (b1 << 16);
    }
}

template <int FMT, int NT>
__global__ void __launch_bounds__(256) k_bs_prep(TcArgs a) {
    grid_dep_wait();  // programmatic dependent launch: the kernel ahead has completed
    grid_dep_trigger();
    constexpr bool BF = FMT == URB_FMT_BF16;
    // 32-column blocks per stage; code words per lane per term.
    constexpr int KBS = FMT == URB_FMT_MXFP4 ? 8 : (FMT == URB_FMT_MXFP8 ? 4 : 2);
    constexpr int QW = FMT == URB_FMT_MXFP4 ? 1 : (FMT == URB_FMT_MXFP8 ? 2 : 4);
    constexpr int RT = bs_rows_per_tok(FMT), TT = NT;
    __shared__ int skip;
    if (threadIdx.x == 0) skip = (a.status && *a.status) ? 1 : 0;
    __syncthreads();
    if (skip) return;
    const long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    const long long item = tid >> 2;
    const int part = int(tid & 3);
    const int nkb = a.ks * KBS;
    bool valid = item < (long long)a.nrows * nkb;
    const int row = valid ? int(item / nkb) : 0, kb = valid ? int(item % nkb) : 0;
    const bool shared_dst = a.inv && a.shared_col0 >= 0 && row >= a.shared_row0 &&
                            row < a.shared_row0 + a.shared_rows;
    if (valid) {
        // Rows that feed no column of this rank (expert-parallel shards) are not loaded.
        if (a.inv) {
            bool any = shared_dst;
            for (int d = 0; d < a.top_k && !any; ++d) any = a.inv[row * a.top_k + d] >= 0;
            valid = any;
        } else if (a.nvalid) {
            valid = row < *a.nvalid || row >= a.routed_cols;
        }
    }
    float r[8];
    const int c0 = kb * 32 + part * 8;
    bool bad = false;
    if (valid) {
        const float *p = a.src_ranks ? a.src_ranks[row / a.rows_per_rank] +
                                           size_t(row % a.rows_per_rank) * a.src_stride
                                     : a.src + size_t(row) * a.src_stride;
        if (!a.swiglu && (a.src_stride & 3) == 0 && c0 + 8 <= a.cols) {
            const float4 v0 = *reinterpret_cast<const float4 *>(p + c0);
            const float4 v1 = *reinterpret_cast<const float4 *>(p + c0 + 4);
            r[0] = v0.x; r[1] = v0.y; r[2] = v0.z; r[3] = v0.w;
            r[4] = v1.x; r[5] = v1.y; r[6] = v1.z; r[7] = v1.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int c = c0 + i;
                float v = 0.0f;
                if (c < a.cols) v = a.swiglu ? silu_f(p[c]) * p[a.cols + c] : p[c];
                r[i] = v;
            }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) bad |= !isfinite(r[i]);
        if (bad) set_status(a.status, URB_ERR_NONFINITE);
    }
    if (!valid || bad) {
#pragma unroll
        for (int i = 0; i < 8; ++i) r[i] = 0.0f;
    }
    if (a.sim128) {
        // E4M3 activation simulation per 128 columns: four 32-column blocks, i.e. 16 lanes
        // (a row's blocks start on a multiple of four, so the groups never straddle rows).
        float m = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(r[i]));
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (a.sim128 == 1) {
            const float scale = num_e4m3_scale(m);
#pragma unroll
            for (int i = 0; i < 8; ++i) r[i] = num_e4m3_sim(r[i], scale);
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) r[i] = num_e4m3_sim_fine(r[i], m);
        }
    }
    uint32_t q[TT][QW];
    int sb[TT];
#pragma unroll
    for (int t = 0; t < TT; ++t) {
        if constexpr (BF) {
            make_term8_bf16(r, q[t]);
            sb[t] = 0;
        } else {
            sb[t] = make_term8<FMT>(r, q[t]);
        }
    }
    if (!valid) return;
    const int ks = kb / KBS, kbs = kb % KBS;
    const int ndst = a.inv ? a.top_k + (shared_dst ? 1 : 0) : 1;
    // Destinations in batches: the column indices, then their slots, are loaded together (two
    // round trips per batch instead of two per destination).
    constexpr int kDb = 4;
    for (int d0 = 0; d0 < ndst; d0 += kDb) {
        int cols[kDb];
        BsSlot sl[kDb];
#pragma unroll
        for (int j = 0; j < kDb; ++j) {
            const int d = d0 + j;
            cols[j] = d >= ndst ? -1
                                : (a.inv ? (d < a.top_k ? a.inv[row * a.top_k + d]
                                                        : a.shared_col0 + (row - a.shared_row0))
                                         : row);
        }
#pragma unroll
        for (int j = 0; j < kDb; ++j)
            if (cols[j] >= 0) sl[j] = a.slots[cols[j]];
#pragma unroll
        for (int j = 0; j < kDb; ++j) {
            if (cols[j] < 0) continue;
            const BsSlot S = sl[j];
            uint8_t *stage = a.bbuf + S.base + (long long)ks * bs_bstage_bytes(FMT, S.n);
#pragma unroll
            for (int t = 0; t < TT; ++t) {
                const int R = S.slot * RT + t;  // MMA row within the stage
                uint8_t *rowp = stage + (R >> 3) * 1024 + (R & 7) * 128;
                if constexpr (BF) {
                    // The lane's 8 columns are one 16-byte chunk of the 128-byte row.
                    const int ch = 4 * kbs + part;
                    *reinterpret_cast<uint4 *>(rowp + ((ch ^ (R & 7)) << 4)) =
                        make_uint4(q[t][0], q[t][1 % QW], q[t][2 % QW], q[t][3 % QW]);
                    continue;
                } else if (FMT == URB_FMT_MXFP4) {
                    *reinterpret_cast<uint32_t *>(rowp + ((kbs ^ (R & 7)) << 4) + 4 * part) = q[t][0];
                } else {
                    const int ch = 2 * kbs + (part >> 1);
                    *reinterpret_cast<uint2 *>(rowp + ((ch ^ (R & 7)) << 4) + 8 * (part & 1)) =
                        make_uint2(q[t][0], q[t][QW - 1]);
                }
                if (part == 0)
                    stage[S.n * 128 + 512 * (kbs >> 2) + 16 * (R & 31) + 4 * (R >> 5) + (kbs & 3)] = uint8_t(sb[t]);
            }
        }
    }
}

// Repack of the reference layout into the bs layout.  One thread per (tile, row): 128 payload
// bytes (swizzled 16-byte chunks) and the row's scale bytes.
template <int FMT>
__global__ void k_repack_bs(const uint8_t *values, const uint8_t *scales, size_t rows, size_t cols,
                            size_t scale_cols, size_t block_rows, size_t block_cols, int mts,
                            int ks_n, uint8_t *out) {
    const size_t id = blockIdx.x * size_t(blockDim.x) + threadIdx.x;
    if (id >= size_t(mts) * ks_n * 128) return;
    const int r = int(id & 127);
    const size_t tile = id >> 7;  // K-stage major: tile (mt, ks) at ks * mts + mt
    const size_t mt = tile % mts;
    const int ks = int(tile / mts);
    const size_t row = mt * 128 + r;
    constexpr int TB = bs_tile_bytes(FMT);
    constexpr int KBS = FMT == URB_FMT_MXFP4 ? 8 : 4;
    uint8_t *t = out + tile * TB;
    uint8_t *rowp = t + (r >> 3) * 1024 + (r & 7) * 128;
    const size_t c0 = size_t(ks) * bs_stage_cols(FMT);
    for (int ch = 0; ch < 8; ++ch) {
        uint32_t wv[4] = {0, 0, 0, 0};
        for (int i = 0; i < 16; ++i) {
            const int byte = ch * 16 + i;
            uint32_t b;
            if (FMT == URB_FMT_MXFP4) {
                const size_t c = c0 + 2 * byte;
                const size_t row_bytes = (cols + 1) / 2;
                uint32_t lo = 0, hi = 0;
                if (row < rows && c < cols) lo = values[row * row_bytes + c / 2] & 0x0f;
                if (row < rows && c + 1 < cols) hi = values[row * row_bytes + c / 2] >> 4;
                b = lo | (hi << 4);
            } else {
                const size_t c = c0 + byte;
                b = (row < rows && c < cols) ? values[row * cols + c] : 0;
            }
            wv[i >> 2] |= b << (8 * (i & 3));
        }
        *reinterpret_cast<uint4 *>(rowp + ((ch ^ (r & 7)) << 4)) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
    }
    for (int kb = 0; kb < KBS; ++kb) {
        const size_t c = c0 + 32 * size_t(kb);
        uint8_t s = 127;
        if (row < rows && c < cols)
            s = FMT == URB_FMT_MXFP4 ? scales[row * scale_cols + c / 32]
                                     : scales[(row / block_rows) * scale_cols + c / block_cols];
        t[16384 + 512 * (kb >> 2) + 16 * (r & 31) + 4 * (r >> 5) + (kb & 3)] = s;
    }
}

template <int FMT, int NT>
int launch_bs_prep_t(Ctx *ctx, const TcArgs &a, cudaStream_t st) {
    static_assert(NT <= bs_rows_per_tok(FMT), "terms fit in a token's MMA rows");
    constexpr int KBS = FMT == URB_FMT_MXFP4 ? 8 : (FMT == URB_FMT_MXFP8 ? 4 : 2);
    const long long threads = (long long)a.nrows * a.ks * KBS * 4;
    if (threads > 0) {
        prof_begin(ctx, URB_K_PREP, st);
        auto prep = k_bs_prep<FMT, NT>;
        URB_LAUNCH_DEP(prep, unsigned((threads + 255) / 256), 256, 0, st, a);
        prof_end(ctx, st);
        URB_CUDA(ctx, cudaGetLastError());
    }
    return URB_OK;
}

template <int FMT, int NT>
int launch_bs_t(Ctx *ctx, const TcArgs &a, int kind, cudaStream_t st) {
    if (!a.skip_prep) {
        const int rc = launch_bs_prep_t<FMT, NT>(ctx, a, st);
        if (rc) return rc;
    }
    auto k = a.pair == 1 ? k_bs_grouped<FMT, 1, NT>
                         : (a.pair == 2 ? k_bs_grouped<FMT, 2, NT> : k_bs_grouped<FMT, 0, NT>);
    URB_CUDA(ctx, cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBs));
    prof_begin(ctx, kind, st);
    URB_LAUNCH_DEP(k, ctx->num_sms, kThreadsBs, kSmemBs, st, a);
    prof_end(ctx, st);
    URB_CUDA(ctx, cudaGetLastError());
    return URB_OK;
}

}  // namespace

int launch_tc_grouped(Ctx *ctx, int fmt, const TcArgs &a, int kind, cudaStream_t st) {
    if (fmt == URB_FMT_MXFP4 && a.full_terms)
        return launch_bs_t<URB_FMT_MXFP4, bs_rows_per_tok(URB_FMT_MXFP4)>(ctx, a, kind, st);
    if (fmt == URB_FMT_MXFP4) return launch_bs_t<URB_FMT_MXFP4, bs_terms(URB_FMT_MXFP4)>(ctx, a, kind, st);
    if (fmt == URB_FMT_MXFP8) return launch_bs_t<URB_FMT_MXFP8, bs_terms(URB_FMT_MXFP8)>(ctx, a, kind, st);
    if (fmt == URB_FMT_BF16) {
        if (a.sim128) return set_error(ctx, URB_ERR_UNSUPPORTED, "tc pass: BF16 takes no E4M3 simulation");
        return launch_bs_t<URB_FMT_BF16, bs_terms(URB_FMT_BF16)>(ctx, a, kind, st);
    }
    return set_error(ctx, URB_ERR_UNSUPPORTED, "tc pass: format");
}

int launch_tc_prep(Ctx *ctx, int fmt, const TcArgs &a, cudaStream_t st) {
    if (fmt == URB_FMT_MXFP4 && a.full_terms)
        return launch_bs_prep_t<URB_FMT_MXFP4, bs_rows_per_tok(URB_FMT_MXFP4)>(ctx, a, st);
    if (fmt == URB_FMT_MXFP4) return launch_bs_prep_t<URB_FMT_MXFP4, bs_terms(URB_FMT_MXFP4)>(ctx, a, st);
    if (fmt == URB_FMT_MXFP8) return launch_bs_prep_t<URB_FMT_MXFP8, bs_terms(URB_FMT_MXFP8)>(ctx, a, st);
    if (fmt == URB_FMT_BF16 && !a.sim128) return launch_bs_prep_t<URB_FMT_BF16, bs_terms(URB_FMT_BF16)>(ctx, a, st);
    return set_error(ctx, URB_ERR_UNSUPPORTED, "tc prep: format");
}

int repack_tc(Ctx *ctx, Mat *m, cudaStream_t st) {
    const bool ok = (m->format == URB_FMT_MXFP4 && m->group_size == 32) ||
                    (m->format == URB_FMT_MXFP8 && m->block_cols % 32 == 0);
    if (!ok) return URB_OK;
    m->tc_mts = int((m->rows + 127) / 128);
    m->tc_ks = int((m->cols + bs_stage_cols(m->format) - 1) / bs_stage_cols(m->format));
    const int TB = bs_tile_bytes(m->format);
    URB_CUDA(ctx, cudaMallocAsync((void **)&m->tc_tiles, size_t(m->tc_mts) * m->tc_ks * TB, st));
    const size_t threads = size_t(m->tc_mts) * m->tc_ks * 128;
    const unsigned blocks = unsigned((threads + 255) / 256);
    const uint8_t *v = static_cast<const uint8_t *>(m->raw_values);
    if (m->format == URB_FMT_MXFP4) {
        const size_t sc = (m->cols + m->group_size - 1) / m->group_size;
        k_repack_bs<URB_FMT_MXFP4><<<blocks, 256, 0, st>>>(v, m->raw_scales, m->rows, m->cols, sc,
                                                          1, 32, m->tc_mts, m->tc_ks, m->tc_tiles);
    } else {
        const size_t sc = (m->cols + m->block_cols - 1) / m->block_cols;
        k_repack_bs<URB_FMT_MXFP8><<<blocks, 256, 0, st>>>(v, m->raw_scales, m->rows, m->cols, sc,
                                                          m->block_rows, m->block_cols, m->tc_mts,
                                                          m->tc_ks, m->tc_tiles);
    }
    URB_CUDA(ctx, cudaGetLastError());
    return URB_OK;
}

}  // namespace urb
