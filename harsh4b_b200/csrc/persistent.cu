// Persistent decode step: one cooperative kernel per token, one CTA per SM.
//
// Same arithmetic as the kernel chain in decode.cu (the same prologues,
// tile math, epilogues and attention order), organised so the weight stream
// never stops at a phase boundary:
//
//   * the producer warp of each CTA walks that SM's rows of every weight
//     matrix of the token in phase order (per layer qkv, o, gate/up, down;
//     then the LM head) and streams them through a 14-slot shared-memory
//     ring (slots of up to 16 KB) with 1-D bulk copies, waiting only for
//     free slots;
//   * seven consumer warps run the phases: poll the phase's input, quantise
//     it (prologue), consume this phase's ring tiles (each slot is owned by
//     one warp), write the outputs (epilogue);
//   * every value one CTA hands to another is a tagged 64-bit exchange word
//     {tag, fp32}; readers poll the words themselves until the tag of this
//     launch and handoff appears (no flags, no fences, no clearing);
//   * attention runs on the first kv_heads * S CTAs (S splits per kv head,
//     chosen per token from the context length); split 0 of each kv head
//     merges the splits in split order.
//
// The ring covers a few microseconds of this SM's share of HBM bandwidth,
// so the producer keeps loading the next phases' weights while consumers
// wait on a dependency. Every wait is bounded; a CTA that gives up sets the
// status word and every other CTA then stops at its next wait.
#include <cstdlib>

#include "common.cuh"

namespace h4b {

// 7 consumer warps + 1 producer warp: two warps per SM sub-partition, so a
// thread may hold up to 255 registers (9 warps would cap it at 168).
constexpr int kMkWarps = 7;  // consumer warps
constexpr int kMkConsumers = kMkWarps * 32;
constexpr int kRmsLanes = 256;  // lanes of the RMSNorm reduction order (see mk_prologue_rms_g)
static_assert(kMkConsumers >= kRmsLanes - 32 && kMkConsumers <= kRmsLanes, "RMS lane map");
constexpr int kMkThreads = kMkConsumers + 32;
constexpr int kMkMaxSlotBytes = 16384;
constexpr int kMkStages = 14;  // a multiple of kMkWarps: each ring slot has one owning warp
constexpr int kMkMaxStages = kMkStages;
constexpr int kMkMaxHidden = 4096;  // RMSNorm inputs kept in registers (2 groups of 8 per lane)
constexpr int kMkMaxWidth = 16384;

enum { SEG_QKV = 0, SEG_O = 1, SEG_GATE_UP = 2, SEG_DOWN = 3 };

constexpr int kMkMaxCtas = 1024;   // exchange words sized for up to this many CTAs
constexpr int kMkSplitCap = 64;    // attention splits per kv head at most

// Tagged exchange words (state->exchange): every value one CTA hands to
// others is a 64-bit word {tag, fp32 payload}. Offsets in words; every
// region starts on a 16-byte boundary.
struct XLayout {
    long long x_o, x_down, qkv, part, att, att_max, act, act_max, keys, gen, total;
};

__host__ __device__ inline long long round4(long long n) { return (n + 3) & ~3ll; }

__host__ __device__ inline XLayout x_layout(const h4b_model& m) {
    const long long H = m.hidden, Q = static_cast<long long>(m.heads) * m.head_dim;
    const long long KV = static_cast<long long>(m.kv_heads) * m.head_dim;
    const long long groups = m.kv_heads > 0 ? m.heads / m.kv_heads : 0;
    XLayout x;
    x.x_o = 0;                                  // x after the o residual, [H]
    x.x_down = x.x_o + round4(H);               // x after the down residual, [H]
    x.qkv = x.x_down + round4(H);               // q, k, v projections, [Q + 2 KV]
    x.part = x.qkv + round4(Q + 2 * KV);        // split partials [kv][splits][groups][kPartialStride]
    x.att = x.part + static_cast<long long>(m.kv_heads) * kMkSplitCap * groups * kPartialStride;
    x.att_max = x.att + round4(Q);              // attended [Q], then its absmax per kv head
    x.act = x.att_max + round4(m.kv_heads);     // SwiGLU output [I], then its absmax per CTA
    x.act_max = x.act + round4(m.intermediate);
    x.keys = x.act_max + kMkMaxCtas;            // per-CTA argmax key (two words)
    x.gen = x.keys + 2 * kMkMaxCtas;            // per-CTA launch counters (never cleared)
    x.total = x.gen + kMkMaxCtas;
    return x;
}

// Tags: launch generation g (per-CTA counters that every launch advances, so
// all CTAs agree without any clearing) and 6 handoffs per layer plus the
// final one. A stale word always carries an older tag.
enum { TAG_QKV = 0, TAG_PART = 1, TAG_ATT = 2, TAG_XO = 3, TAG_ACT = 4, TAG_XDOWN = 5, kTagsPerLayer = 6 };
__host__ __device__ inline uint32_t mk_tag_base(uint32_t gen, int layers) {
    return 1u + gen * static_cast<uint32_t>(kTagsPerLayer * layers + 2);
}

struct MkArgs {
    h4b_model m;
    h4b_state s;
    XLayout x;
    int stages;
    int slot_bytes;        // ring slot size (a tile is at most one slot)
    int attn_chunk;        // target tokens per attention split
    int max_splits;        // splits per kv head at most
    int stage_splits;      // splits whose partials fit the K/V staging area
    int xq_bytes, rows_cap;
};

struct Seg {
    const uint8_t* w;
    const float* ws;
    int width, kb, r0, nrows, tile_rows, ntiles;
};

// Where one CTA's rows of each kind of GEMV segment lie: per kind (qkv, o,
// gate/up, down, LM head) the first row, the row count, rows per ring tile
// and the tile count. Computed once per launch by mk_geometry, so the
// per-segment code holds no divisions.
struct SegGeo {
    int r0, nrows, tile_rows, ntiles;
};
constexpr int kSegKinds = 5;
static_assert(kSegKinds * sizeof(SegGeo) <= 128, "geometry table region");

__device__ __noinline__ void mk_geometry(const MkArgs& a, int cta, int nctas, SegGeo* geo) {
    const h4b_model& m = a.m;
    const int Q = m.heads * m.head_dim, KV = m.kv_heads * m.head_dim;
    const int rows[kSegKinds] = {Q + 2 * KV, m.hidden, 2 * m.intermediate, m.hidden, m.vocab};
    const int kb[kSegKinds] = {m.hidden / 2, Q / 2, m.hidden / 2, m.intermediate / 2, m.hidden / 2};
    for (int k = 0; k < kSegKinds; ++k) {
        const int align = k == SEG_GATE_UP ? 2 * kSwigluBlock : 1;
        const uint32_t units = static_cast<uint32_t>(rows[k] / align);
        // units * (cta + 1) < 2^32: the host checks vocab * CTAs
        const int u0 = static_cast<int>(units * static_cast<uint32_t>(cta) / static_cast<uint32_t>(nctas));
        const int u1 = static_cast<int>(units * static_cast<uint32_t>(cta + 1) / static_cast<uint32_t>(nctas));
        SegGeo gk;
        gk.r0 = u0 * align;
        gk.nrows = (u1 - u0) * align;
        // Fewest rounds of kMkWarps tiles that fit a ring slot, then rows
        // spread evenly over those tiles, so no warp has a short last round
        // while the others idle.
        const int max_rows = max(1, a.slot_bytes / kb[k]);
        const int rounds = ((gk.nrows + max_rows - 1) / max_rows + kMkWarps - 1) / kMkWarps;
        const int tiles = max(1, min(rounds * kMkWarps, gk.nrows));
        gk.tile_rows = max(1, (gk.nrows + tiles - 1) / tiles);
        gk.ntiles = (gk.nrows + gk.tile_rows - 1) / gk.tile_rows;
        geo[k] = gk;
    }
}

// Rows of GEMV segment g (4 per layer, then the LM head) that this CTA owns.
__device__ __forceinline__ Seg mk_segment(const MkArgs& a, const SegGeo* geo, int g) {
    const h4b_model& m = a.m;
    const int H = m.hidden, I = m.intermediate;
    const int Q = m.heads * m.head_dim, KV = m.kv_heads * m.head_dim;
    const int kind = g == 4 * m.layers ? 4 : (g & 3);
    const size_t l = static_cast<size_t>(g >> 2);
    Seg s;
    switch (kind) {
        case SEG_QKV:
            s.width = H;
            s.w = m.w_qkv + l * (Q + 2 * KV) * (H / 2);
            s.ws = m.s_qkv + l * (Q + 2 * KV);
            break;
        case SEG_O:
            s.width = Q;
            s.w = m.w_o + l * H * (Q / 2);
            s.ws = m.s_o + l * H;
            break;
        case SEG_GATE_UP:
            s.width = H;
            s.w = m.w_gate_up + l * 2 * I * (H / 2);
            s.ws = m.s_gate_up + l * 2 * I;
            break;
        case SEG_DOWN:
            s.width = I;
            s.w = m.w_down + l * H * (I / 2);
            s.ws = m.s_down + l * H;
            break;
        default:
            s.width = H;
            s.w = m.w_embed;
            s.ws = m.s_embed;
            break;
    }
    s.kb = s.width >> 1;
    const SegGeo gk = geo[kind];
    s.r0 = gk.r0;
    s.nrows = gk.nrows;
    s.tile_rows = gk.tile_rows;
    s.ntiles = gk.ntiles;
    return s;
}

// The consumers' stop decision: any consumer thread may report a failure
// (`failed`); flags[0] also carries stop requests from any warp, the
// producer included. Thread 0 snapshots flags[0] into flags[1] between two
// barriers, so every consumer thread takes the same branch and none is left
// waiting at a later named barrier.
__device__ bool mk_stop(int* flags, bool failed = false) {
    if (failed) atomicOr(&flags[0], 1);
    named_sync(1, kMkConsumers);
    if (threadIdx.x == 0) flags[1] = *reinterpret_cast<volatile int*>(&flags[0]);
    named_sync(1, kMkConsumers);
    return flags[1] != 0;
}

// Polls the 8-word groups lane_id + k * 256 (k < G, < groups) of exchange
// words until each carries `tag`; leaves the payloads in v. All loads of a
// round are issued before any is checked, so a round costs one L2 round
// trip. On timeout sets the CTA stop flag (values are then zero).
template <int G>
__device__ void mk_poll_lane(const unsigned long long* w, int lane_id, int groups, uint32_t tag, float v[G][8],
                             int* flags) {
    unsigned pending = 0;
#pragma unroll
    for (int k = 0; k < G; ++k)
        if (lane_id + k * kRmsLanes < groups) pending |= 1u << k;
    PollClock clk;
    while (pending) {
        ulonglong2 raw[G][4];
#pragma unroll
        for (int k = 0; k < G; ++k) {
            if (pending & (1u << k)) {
                const unsigned long long* p = w + 8 * (lane_id + k * kRmsLanes);
#pragma unroll
                for (int j = 0; j < 4; ++j) raw[k][j] = ll_load2(p + 2 * j);
            }
        }
#pragma unroll
        for (int k = 0; k < G; ++k) {
            if (!(pending & (1u << k))) continue;
            bool ok = true;
#pragma unroll
            for (int j = 0; j < 4; ++j) ok = ok && ll_tag(raw[k][j].x) == tag && ll_tag(raw[k][j].y) == tag;
            if (ok) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    v[k][2 * j] = ll_value(raw[k][j].x);
                    v[k][2 * j + 1] = ll_value(raw[k][j].y);
                }
                pending &= ~(1u << k);
            }
        }
        if (pending && poll_expired(clk)) {
            atomicOr(&flags[0], 1);
#pragma unroll
            for (int k = 0; k < G; ++k)
                if (pending & (1u << k))
#pragma unroll
                    for (int e = 0; e < 8; ++e) v[k][e] = 0.f;
            break;
        }
    }
}

// Polls one exchange word per thread (index tid + k * kMkConsumers < n) and
// returns the max of the payloads it saw (0 when it holds none).
__device__ float mk_poll_max(const unsigned long long* w, int n, uint32_t tag, int* flags) {
    float mx = 0.f;
    #pragma unroll 1
    for (int i = threadIdx.x; i < n; i += kMkConsumers) {
        PollClock clk;
        unsigned long long word = ll_load(w + i);
        while (ll_tag(word) != tag) {
            if (poll_expired(clk)) {
                atomicOr(&flags[0], 1);
                break;
            }
            word = ll_load(w + i);
        }
        mx = fmaxf(mx, ll_tag(word) == tag ? ll_value(word) : 0.f);
    }
    return mx;
}

// The RMSNorm sum of squares is defined over 256 lanes (the GEMV kernel's
// consumer threads, which the CPU oracle follows): lane p sums groups
// p, p + 256, ... of 8 values with fmaf, each warp of lanes is summed with a
// butterfly, and the 8 warp totals are added in order. Consumer thread t
// computes lane t; warp 0 also computes lanes 224..255 (lane-warp 7).

// RMSNorm + absmax quantisation of x (n <= G * 8 * 256) into xq, in the same
// order as the GEMV kernel's prologue; returns the dequant scale. x is the
// embedding row in shared memory (xs) or exchange words carrying `tag`.
template <int G>
__device__ float mk_prologue_rms_g(const float* xs, const unsigned long long* xw, uint32_t tag, const float* gamma_s,
                                   int n, float eps, int8_t* xq, float* red, int* flags, int trace_ev) {
    const int tid = threadIdx.x, warp = tid >> 5;
    const int groups = n >> 3;
    const bool extra = tid + kMkConsumers < kRmsLanes;  // warp 0: also lane tid + kMkConsumers
    float v[2][G][8];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int lane_id = tid + r * kMkConsumers;
        if (r == 1 && !extra) break;
        if (xw) {
            mk_poll_lane<G>(xw, lane_id, groups, tag, v[r], flags);
            if (trace_ev >= 0) H4B_TRACE_ANY(trace_ev);
        } else {
#pragma unroll
            for (int k = 0; k < G; ++k) {
                const int g = lane_id + k * kRmsLanes;
                if (g < groups) load8(xs + 8 * g, v[r][k]);
            }
        }
    }
    float ss[2] = {0.f, 0.f};
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int lane_id = tid + r * kMkConsumers;
#pragma unroll
        for (int k = 0; k < G; ++k) {
            if ((r == 0 || extra) && lane_id + k * kRmsLanes < groups) {
#pragma unroll
                for (int e = 0; e < 8; ++e) ss[r] = __fmaf_rn(v[r][k][e], v[r][k][e], ss[r]);
            }
        }
    }
    const float w0 = warp_sum(ss[0]);
    const float w1 = warp_sum(ss[1]);  // meaningful in warp 0 only
    if ((tid & 31) == 0) {
        red[warp] = w0;
        if (warp == 0) red[kRmsLanes / 32 - 1] = w1;
    }
    async_copy_wait_prior<1>();  // gamma_s and the segment's scales (the newer group is attention's K/V)
    named_sync(1, kMkConsumers);
    float total = 0.f;
    for (int w = 0; w < kRmsLanes / 32; ++w) total += red[w];
    // (no barrier: the maximum below goes to red[16..], and red[0..7] is
    // next written after the closing barrier)
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(n)), eps)));
    float local = 0.f;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int lane_id = tid + r * kMkConsumers;
#pragma unroll
        for (int k = 0; k < G; ++k) {
            const int g = lane_id + k * kRmsLanes;
            if ((r == 0 || extra) && g < groups) {
                float gm[8];
                load8(gamma_s + 8 * g, gm);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    v[r][k][e] = __fmul_rn(__fmul_rn(v[r][k][e], inv), gm[e]);
                    local = fmaxf(local, fabsf(v[r][k][e]));
                }
            }
        }
    }
    const float m = group_max_open(local, red + 16, kMkWarps, 1);  // closed by the barrier at the end
    const float qs = quant_multiplier(m);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int lane_id = tid + r * kMkConsumers;
#pragma unroll
        for (int k = 0; k < G; ++k) {
            const int g = lane_id + k * kRmsLanes;
            if ((r == 0 || extra) && g < groups) {
                int q[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) q[e] = quantize_one(v[r][k][e], qs);
                store_group(xq, g, q);
            }
        }
    }
    zero_xq_tail(xq, n, tid, kMkConsumers);
    named_sync(1, kMkConsumers);
    return dequant_scale(m);
}

__device__ float mk_prologue_rms(const float* xs, const unsigned long long* xw, uint32_t tag, const float* gamma_s,
                                 int n, float eps, int8_t* xq, float* red, int* flags, int trace_ev = -1) {
    return mk_prologue_rms_g<kMkMaxHidden / (8 * kRmsLanes)>(xs, xw, tag, gamma_s, n, eps, xq, red, flags, trace_ev);
}

// Quantisation of n exchange words carrying `tag` with the absmax over the
// nmax partial maxima its producers published (also tagged `tag`). Each
// thread loads its maxima word(s) and all its 8-word groups
// (g = tid + k * kMkConsumers, k < kMkQuantGroups) in every polling round,
// so the whole handoff costs one L2 round trip once the data is there.
constexpr int kMkQuantGroups = 6;  // covers 6 * 8 * 224 = 10752 values
__device__ float mk_prologue_quant(const unsigned long long* vw, const unsigned long long* maxw, int nmax, uint32_t tag,
                                   int n, int8_t* xq, float* red, int* flags, int trace_ev = -1) {
    const int tid = threadIdx.x;
    const int groups = n >> 3;
    unsigned pending = 0;
#pragma unroll
    for (int k = 0; k < kMkQuantGroups; ++k)
        if (tid + k * kMkConsumers < groups) pending |= 1u << k;
    const bool has_max = tid < nmax;  // nmax <= kMkConsumers (checked on the host)
    bool max_done = !has_max;
    float mx = 0.f;
    ulonglong2 raw[kMkQuantGroups][4];  // the words themselves hold the values once their tags check
    PollClock clk;
    while (pending || !max_done) {
        unsigned long long mword = 0;
        if (!max_done) mword = ll_load(maxw + tid);
#pragma unroll
        for (int k = 0; k < kMkQuantGroups; ++k) {
            if (pending & (1u << k)) {
                const unsigned long long* p = vw + 8 * (tid + k * kMkConsumers);
#pragma unroll
                for (int j = 0; j < 4; ++j) raw[k][j] = ll_load2(p + 2 * j);
            }
        }
        if (!max_done && ll_tag(mword) == tag) {
            mx = ll_value(mword);
            max_done = true;
        }
#pragma unroll
        for (int k = 0; k < kMkQuantGroups; ++k) {
            if (!(pending & (1u << k))) continue;
            bool ok = true;
#pragma unroll
            for (int j = 0; j < 4; ++j) ok = ok && ll_tag(raw[k][j].x) == tag && ll_tag(raw[k][j].y) == tag;
            if (ok) pending &= ~(1u << k);
        }
        if ((pending || !max_done) && poll_expired(clk)) {
            atomicOr(&flags[0], 1);
            break;
        }
    }
    if (trace_ev >= 0) H4B_TRACE_ANY(trace_ev + 1);
    const float m = group_max_open(mx, red, kMkWarps, 1);  // closed by the barrier at the end
    const float qs = quant_multiplier(m);
#pragma unroll
    for (int k = 0; k < kMkQuantGroups; ++k) {
        const int g = tid + k * kMkConsumers;
        if (g < groups) {
            int q[8];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                q[2 * j] = quantize_one(ll_value(raw[k][j].x), qs);
                q[2 * j + 1] = quantize_one(ll_value(raw[k][j].y), qs);
            }
            store_group(xq, g, q);
        }
    }
    zero_xq_tail(xq, n, tid, kMkConsumers);
    named_sync(1, kMkConsumers);
    return dequant_scale(m);
}

// This CTA's tiles of one GEMV segment: int32 row sums into acc_s.
template <int SLOTS, int RB>
__device__ void mk_tiles(const Seg& sg, uint32_t seq0, int stages, int slot_bytes, const uint8_t* ring, uint64_t* full,
                         uint64_t* empty, const int8_t* xq, int32_t* acc_s, int* flags, int trace_ev) {
    constexpr bool kXReg = SLOTS <= kMaxRegSlots;
    constexpr int kXSlots = kXReg ? SLOTS : 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int chunks = sg.width >> 5;
    uint4 xa[kXSlots], xb[kXSlots];
    int bias = 0;
#pragma unroll
    for (int j = 0; j < SLOTS; ++j) {
        const int c = lane + 32 * j;
        if (c < chunks) {
            const uint4 va = *reinterpret_cast<const uint4*>(xq + 32 * c);
            const uint4 vb = *reinterpret_cast<const uint4*>(xq + 32 * c + 16);
            const uint32_t words[8] = {va.x, va.y, va.z, va.w, vb.x, vb.y, vb.z, vb.w};
#pragma unroll
            for (int e = 0; e < 8; ++e) bias = __dp4a(static_cast<int>(words[e]), 0x01010101, bias);
            if constexpr (kXReg) {
                xa[j] = va;
                xb[j] = vb;
            }
        } else if constexpr (kXReg) {
            xa[j] = make_uint4(0, 0, 0, 0);
            xb[j] = make_uint4(0, 0, 0, 0);
        }
    }
    bias *= -8;
    if (trace_ev >= 0 && threadIdx.x == 0) H4B_TRACE_ANY(trace_ev);
    for (int t = warp; t < sg.ntiles; t += kMkWarps) {
        const uint32_t gseq = seq0 + t;
        const int slot = gseq % stages;
        if (*reinterpret_cast<volatile int*>(&flags[0])) break;
        if (!mbar_wait(&full[slot], (gseq / stages) & 1)) {
            atomicOr(&flags[0], 1);
            break;
        }
        if (lane == 0 && gseq >= 40 && gseq < 140) H4B_TRACE_ANY(1200 + gseq - 40);
        const uint8_t* tile = ring + static_cast<size_t>(slot) * slot_bytes;
        const int trows = min(sg.tile_rows, sg.nrows - t * sg.tile_rows);
        for (int b0 = 0; b0 < trows; b0 += RB) {
            int total[RB];
            tile_batch<SLOTS, RB, kXReg>(tile, sg.kb, trows, b0, xa, xb, xq, lane, bias, total);
            if (lane == 0) {
#pragma unroll
                for (int i = 0; i < RB; ++i)
                    if (b0 + i < trows) acc_s[t * sg.tile_rows + b0 + i] = total[i];
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        if (lane == 0 && gseq >= 40 && gseq < 140) H4B_TRACE_ANY(1300 + gseq - 40);
    }
    async_copy_wait_prior<1>();   // the segment's row scales (the newer group is attention's K/V)
    named_sync(1, kMkConsumers);  // acc_s complete, scales visible
}

__device__ void mk_run_tiles(const Seg& sg, uint32_t seq0, int stages, int slot_bytes, const uint8_t* ring, uint64_t* full,
                             uint64_t* empty, const int8_t* xq, int32_t* acc_s, int* flags, int trace_ev = -1) {
    const int need = ((sg.width >> 5) + 31) / 32;
    // Three rows per batch where the tile height allows it (more independent
    // work per pass over the activation), else two.
    if (sg.tile_rows % 3 == 0 && need <= 4) {
        if (need <= 3) mk_tiles<3, 3>(sg, seq0, stages, slot_bytes, ring, full, empty, xq, acc_s, flags, trace_ev);
        else mk_tiles<4, 3>(sg, seq0, stages, slot_bytes, ring, full, empty, xq, acc_s, flags, trace_ev);
        return;
    }
    if (need <= 1) mk_tiles<1, 2>(sg, seq0, stages, slot_bytes, ring, full, empty, xq, acc_s, flags, trace_ev);
    else if (need <= 2) mk_tiles<2, 2>(sg, seq0, stages, slot_bytes, ring, full, empty, xq, acc_s, flags, trace_ev);
    else if (need <= 3) mk_tiles<3, 2>(sg, seq0, stages, slot_bytes, ring, full, empty, xq, acc_s, flags, trace_ev);
    else if (need <= 4) mk_tiles<4, 2>(sg, seq0, stages, slot_bytes, ring, full, empty, xq, acc_s, flags, trace_ev);
    else if (need <= 6) mk_tiles<6, 2>(sg, seq0, stages, slot_bytes, ring, full, empty, xq, acc_s, flags, trace_ev);
    else if (need <= 8) mk_tiles<8, 2>(sg, seq0, stages, slot_bytes, ring, full, empty, xq, acc_s, flags, trace_ev);
    else if (need <= 10) mk_tiles<10, 2>(sg, seq0, stages, slot_bytes, ring, full, empty, xq, acc_s, flags, trace_ev);
    else if (need <= 12) mk_tiles<12, 2>(sg, seq0, stages, slot_bytes, ring, full, empty, xq, acc_s, flags, trace_ev);
    else mk_tiles<16, 2>(sg, seq0, stages, slot_bytes, ring, full, empty, xq, acc_s, flags, trace_ev);
}

// Starts the 4-byte async copies of a segment's row scales into sc_s.
__device__ __forceinline__ void mk_fetch_scales(const Seg& sg, float* sc_s) {
    #pragma unroll 1
    for (int i = threadIdx.x; i < sg.nrows; i += kMkConsumers) async_copy4(sc_s + i, sg.ws + sg.r0 + i);
}

// Starts the async copy of an RMSNorm weight (n floats, n % 4 == 0, 16-byte
// aligned) into gamma_s.
__device__ __forceinline__ void mk_fetch_gamma(const float* gamma, float* gamma_s, int n) {
    #pragma unroll 1
    for (int i = threadIdx.x; i < (n >> 2); i += kMkConsumers) async_copy16(gamma_s + 4 * i, gamma + 4 * i);
}

// Starts the async copies of what GEMV segment g itself needs: its row
// scales (into scale buffer g & 1, which segment g - 2 last read) and, for an
// RMSNorm prologue (qkv, gate/up, LM head), the norm weight. Issued before
// the segment's input is polled, so the copies overlap the handoff wait; the
// RMSNorm prologue and the tile loop wait for them before reading.
__device__ __forceinline__ void mk_fetch_own(const MkArgs& a, int g, const SegGeo* geo, float* sc_base,
                                             float* gamma_s) {
    const h4b_model& m = a.m;
    const int H = m.hidden;
    const size_t l = static_cast<size_t>(g >> 2);
    mk_fetch_scales(mk_segment(a, geo, g), sc_base + (g & 1) * a.rows_cap);
    if (g == 4 * m.layers) mk_fetch_gamma(m.norm_final, gamma_s, H);
    else if ((g & 3) == SEG_QKV) mk_fetch_gamma(m.norm_in + l * H, gamma_s, H);
    else if ((g & 3) == SEG_GATE_UP) mk_fetch_gamma(m.norm_post + l * H, gamma_s, H);
}

__device__ __forceinline__ float mk_value(const int32_t* acc_s, const float* sc_s, int i, float act_scale) {
    return __fmul_rn(__fmul_rn(static_cast<float>(acc_s[i]), act_scale), sc_s[i]);
}

// Polls the 4 exchange words of a 128-wide head that lane `lane` holds.
__device__ __forceinline__ bool mk_poll_head(const unsigned long long* w, int lane, uint32_t tag, float4& out) {
    const unsigned long long* p = w + 4 * lane;
    PollClock clk;
    while (true) {
        const ulonglong2 a = ll_load2(p), b = ll_load2(p + 2);
        if (ll_tag(a.x) == tag && ll_tag(a.y) == tag && ll_tag(b.x) == tag && ll_tag(b.y) == tag) {
            out = make_float4(ll_value(a.x), ll_value(a.y), ll_value(b.x), ll_value(b.y));
            return true;
        }
        if (poll_expired(clk)) {
            out = make_float4(0.f, 0.f, 0.f, 0.f);
            return false;
        }
    }
}

// merge_splits over exchange words for long contexts (more splits than one
// staging batch): split 0 from registers, each other split polled in turn.
__device__ float4 mk_merge_direct(const unsigned long long* base, int splits, long long stride, uint32_t tag,
                                  float m0, float l0, float4 o0, int lane, bool& ok) {
    float mmax = -INFINITY;
    #pragma unroll 1
    for (int s = lane; s < splits; s += 32) {
        float mv = m0;
        if (s != 0) {
            PollClock clk;
            unsigned long long w = ll_load(base + s * stride + kHeadDim);
            while (ll_tag(w) != tag) {
                if (poll_expired(clk)) {
                    ok = false;
                    break;
                }
                w = ll_load(base + s * stride + kHeadDim);
            }
            mv = ll_value(w);
        }
        mmax = fmaxf(mmax, mv);
    }
    mmax = warp_max(mmax);
    float l = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    #pragma unroll 1
    for (int s = 0; s < splits; ++s) {
        float ms = m0, ls = l0;
        float4 ov = o0;
        if (s != 0) {
            const unsigned long long* p = base + s * stride;
            PollClock clk;
            while (true) {
                const ulonglong2 a = ll_load2(p + 4 * lane), b = ll_load2(p + 4 * lane + 2);
                const ulonglong2 c = ll_load2(p + kHeadDim);
                const bool good = ll_tag(a.x) == tag && ll_tag(a.y) == tag && ll_tag(b.x) == tag &&
                                  ll_tag(b.y) == tag && ll_tag(c.x) == tag && ll_tag(c.y) == tag;
                if (__all_sync(0xffffffffu, good)) {
                    ov = make_float4(ll_value(a.x), ll_value(a.y), ll_value(b.x), ll_value(b.y));
                    ms = ll_value(c.x);
                    ls = ll_value(c.y);
                    break;
                }
                if (poll_expired(clk)) {
                    ok = false;
                    break;
                }
            }
        }
        if (ls == 0.f) continue;
        const float w = exp_cw(ms - mmax);
        l = __fmaf_rn(ls, w, l);
        acc.x = __fmaf_rn(ov.x, w, acc.x);
        acc.y = __fmaf_rn(ov.y, w, acc.y);
        acc.z = __fmaf_rn(ov.z, w, acc.z);
        acc.w = __fmaf_rn(ov.w, w, acc.w);
    }
    const float inv = __fdiv_rn(1.0f, l);
    return make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
}

// Starts the async copies attention needs before the new token's q/k/v
// exist: the split's first sub-tile of past K/V rows (the new token's row,
// which arrives from registers, is left out) and the q/k norm weights plus
// this position's RoPE row into consts_s ([0, d) q gamma, [d, 2d) k gamma,
// [2d, 2.5d) cos, [2.5d, 3d) sin). From layer 1 on the kernel issues them at
// the top of the qkv segment, so they land while the qkv input is polled.
template <typename KV>
__device__ __forceinline__ void mk_attention_fetch(const MkArgs& a, int l, int h, int split, int splits, int pos,
                                                   KV* ks, KV* vs, float* consts_s) {
    const h4b_model& m = a.m;
    const h4b_state& st = a.s;
    const int d = kHeadDim;
    const int ctx = pos + 1;
    const int chunk = (ctx + splits - 1) / splits;
    const int t0 = min(ctx, split * chunk), t1 = min(ctx, t0 + chunk);
    const float* cs = m.rope_cos + static_cast<long long>(pos) * (d / 2);
    const float* sn = m.rope_sin + static_cast<long long>(pos) * (d / 2);
    const size_t kv_layer = static_cast<size_t>(m.kv_heads) * st.capacity * d;
    const KV* kc = static_cast<const KV*>(st.k_cache) + l * kv_layer + static_cast<size_t>(h) * st.capacity * d;
    const KV* vc = static_cast<const KV*>(st.v_cache) + l * kv_layer + static_cast<size_t>(h) * st.capacity * d;
    const bool owns_new = t0 <= pos && pos < t1;
    if (t0 < t1) stage_subtile<KV>(kc, vc, d, t0, min(kSubTile, t1 - t0), owns_new ? pos : -1, ks, vs, threadIdx.x,
                                   kMkConsumers);
#pragma unroll 1
    for (int i = threadIdx.x; i < 3 * d / 4; i += kMkConsumers) {
        const float* src = i < d / 4 ? m.norm_q + static_cast<size_t>(l) * d + 4 * i
                         : i < d / 2 ? m.norm_k + static_cast<size_t>(l) * d + 4 * (i - d / 4)
                         : i < 5 * d / 8 ? cs + 4 * (i - d / 2)
                                         : sn + 4 * (i - 5 * d / 8);
        async_copy16(consts_s + 4 * i, src);
    }
}

// One attention split (kv head h, split `split` of `splits`) for layer l,
// in the order of gqa_split_kernel. The first sub-tile of past K/V rows and
// the norm/RoPE constants are fetched before the new token's q/k/v are
// polled. Splits other than 0 publish (o, m, l) per q head as exchange
// words; split 0 merges them in split order (merge_splits' arithmetic) and
// publishes the attended heads and their absmax. Returns false if the CTA
// must stop.
template <typename KV>
__device__ bool mk_attention(const MkArgs& a, unsigned long long* xw, uint32_t tbase, int l, int h, int split,
                             int splits, int pos, KV* ks, KV* vs, float* consts_s, float* red, int* flags,
                             bool prefetched) {
    const h4b_model& m = a.m;
    const h4b_state& st = a.s;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int groups = m.heads / m.kv_heads;
    const int d = kHeadDim;
    const int q_size = m.heads * d, kv_size = m.kv_heads * d;
    const bool head_warp = warp < groups;
    const int qh = h * groups + warp;
    const int ctx = pos + 1;
    const int chunk = (ctx + splits - 1) / splits;
    const int t0 = min(ctx, split * chunk), t1 = min(ctx, t0 + chunk);
    const size_t kv_layer = static_cast<size_t>(m.kv_heads) * st.capacity * d;
    KV* kc = static_cast<KV*>(st.k_cache) + l * kv_layer + static_cast<size_t>(h) * st.capacity * d;
    KV* vc = static_cast<KV*>(st.v_cache) + l * kv_layer + static_cast<size_t>(h) * st.capacity * d;
    const bool owns_new = t0 <= pos && pos < t1;
    const uint32_t tag_qkv = tbase + kTagsPerLayer * l + TAG_QKV;
    const uint32_t tag_part = tbase + kTagsPerLayer * l + TAG_PART;
    const uint32_t tag_att = tbase + kTagsPerLayer * l + TAG_ATT;

    if (!prefetched) mk_attention_fetch<KV>(a, l, h, split, splits, pos, ks, vs, consts_s);
    if (l == 1) H4B_TRACE(1500);
    if (l == 2) H4B_TRACE_CTA(16);

    const unsigned long long* qkv = xw + a.x.qkv;
    bool ok = true;
    float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 k_new = q, v_new = q;
    if (head_warp) ok = mk_poll_head(qkv + static_cast<long long>(qh) * d, lane, tag_qkv, q);
    if (owns_new && warp == 0) ok = mk_poll_head(qkv + q_size + static_cast<long long>(h) * d, lane, tag_qkv, k_new) && ok;
    if (owns_new && warp == groups - 1)
        ok = mk_poll_head(qkv + q_size + kv_size + static_cast<long long>(h) * d, lane, tag_qkv, v_new) && ok;
    if (mk_stop(flags, !ok)) {
        async_copy_wait_all();
        return false;
    }
    if (l == 1) H4B_TRACE(1501);
    if (l == 2) H4B_TRACE_CTA(17);
    async_copy_wait_all();
    named_sync(1, kMkConsumers);  // consts_s (and the first sub-tile) landed
    if (head_warp) {
        q = norm_rope_with(q, head_consts(consts_s, consts_s + 2 * d, consts_s + 5 * d / 2, lane), true, true, m.eps,
                           lane);
        *reinterpret_cast<float4*>(consts_s + (3 + warp) * d + 4 * lane) = q;  // this warp's staged q head
    }
    if (owns_new) {
        if (warp == 0) {
            k_new = norm_rope_with(k_new, head_consts(consts_s + d, consts_s + 2 * d, consts_s + 5 * d / 2, lane),
                                   true, true, m.eps, lane);
            store4<KV>(kc + static_cast<long long>(pos) * d + 4 * lane, k_new);
        }
        if (warp == groups - 1) store4<KV>(vc + static_cast<long long>(pos) * d + 4 * lane, v_new);
    }
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(d)));
    float mrun = -INFINITY, l_run = 0.f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    #pragma unroll 1
    for (int base = t0; base < t1; base += kSubTile) {
        const int n = min(kSubTile, t1 - base);
        if (base != t0) {
            named_sync(1, kMkConsumers);  // the previous sub-tile is consumed
            stage_subtile<KV>(kc, vc, d, base, n, owns_new ? pos : -1, ks, vs, threadIdx.x, kMkConsumers);
        }
        if (owns_new && pos >= base && pos < base + n) {
            if (warp == 0) store4<KV>(ks + (pos - base) * kv_row_stride<KV>() + 4 * lane, k_new);
            if (warp == groups - 1) store4<KV>(vs + (pos - base) * kv_row_stride<KV>() + 4 * lane, v_new);
        }
        async_copy_wait_all();
        named_sync(1, kMkConsumers);
        if (l == 1) H4B_TRACE(1502);
    if (l == 2) H4B_TRACE_CTA(18);
#ifdef H4B_PHASE_TRACE
        if (threadIdx.x == 0) g_trace_attn = (l == 1);
#endif
        if (head_warp) attend_subtile<KV>(consts_s + (3 + warp) * d, ks, vs, n, scale, lane, mrun, l_run, o);
    }
    if (l == 1) H4B_TRACE(1503);
    if (l == 2) H4B_TRACE_CTA(19);

    float4 result = make_float4(0.f, 0.f, 0.f, 0.f);
    const long long pstride = kPartialStride;
    unsigned long long* part = xw + a.x.part + static_cast<long long>(h) * kMkSplitCap * groups * pstride;
    if (splits > 1 && split != 0) {
        if (head_warp) {
            unsigned long long* mine = part + (static_cast<long long>(split) * groups + warp) * pstride;
            ll_store2(mine + 4 * lane, o.x, o.y, tag_part);
            ll_store2(mine + 4 * lane + 2, o.z, o.w, tag_part);
            if (lane == 0) ll_store2(mine + kHeadDim, mrun, l_run, tag_part);
        }
        if (l == 2) H4B_TRACE_CTA(22);
        return true;
    }
    if (splits == 1) {
        if (head_warp) {
            const float inv = __fdiv_rn(1.0f, l_run);
            result = make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
        }
    } else if (splits <= a.stage_splits) {
        // Merge in split order (merge_splits' arithmetic), split 0 from
        // registers. The other splits' partials are copied as raw exchange
        // words into the K/V staging area (free once the math is done). Each
        // thread re-copies its own pieces until every word carries tag_part,
        // with no CTA barrier between polling rounds, so a round costs one
        // L2 round trip; one barrier follows once every thread is done.
        constexpr int kPieces = kPartialStride / 2;  // 16-byte pieces per (split, head) partial
        constexpr int kWordPieces = kHeadDim / 2 + 1;  // o and (m, l); the last piece holds 2 pad words
        unsigned long long* stage = reinterpret_cast<unsigned long long*>(ks);  // [split][groups][kPartialStride]
        const int total = (splits - 1) * groups * kWordPieces;  // pieces of the splits other than 0
        named_sync(1, kMkConsumers);  // every head warp is done reading the K/V sub-tile
        bool timed_out = false;
        PollClock clk;
#pragma unroll 1
        for (bool first = true;; first = false) {
#pragma unroll 1
            for (int i = threadIdx.x; i < total; i += kMkConsumers) {
                const int piece = i % kWordPieces, sh = groups + i / kWordPieces;  // sh = split * groups + head
                unsigned long long* dst = stage + static_cast<long long>(sh) * pstride + 2 * piece;
                if (!first && ll_tag(dst[0]) == tag_part && ll_tag(dst[1]) == tag_part) continue;
                async_copy16(dst, part + static_cast<long long>(sh) * pstride + 2 * piece);
            }
            async_copy_wait_all();
            bool stale = false;
#pragma unroll 1
            for (int i = threadIdx.x; i < total; i += kMkConsumers) {
                const int piece = i % kWordPieces, sh = groups + i / kWordPieces;
                const unsigned long long* w = stage + static_cast<long long>(sh) * pstride + 2 * piece;
                stale = stale || ll_tag(w[0]) != tag_part || ll_tag(w[1]) != tag_part;
            }
            if (!stale) break;
            if (poll_expired(clk)) {
                timed_out = true;
                break;
            }
        }
        static_assert(kWordPieces < kPieces, "pad piece");
        if (mk_stop(flags, timed_out)) return false;  // its barrier also publishes every staged piece
        if (head_warp) {
            const unsigned long long* mine = stage + warp * pstride;
            float mm = -INFINITY;
            #pragma unroll 1
            for (int s = lane; s < splits; s += 32)
                mm = fmaxf(mm, s == 0 ? mrun : ll_value(mine[static_cast<long long>(s) * groups * pstride + kHeadDim]));
            mm = warp_max(mm);
            float lsum = 0.f;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            #pragma unroll 1
            for (int s = 0; s < splits; ++s) {
                const unsigned long long* w = mine + static_cast<long long>(s) * groups * pstride;
                const float ls = s == 0 ? l_run : ll_value(w[kHeadDim + 1]);
                if (ls == 0.f) continue;
                const float ms = s == 0 ? mrun : ll_value(w[kHeadDim]);
                const float4 ov = s == 0 ? o
                                         : make_float4(ll_value(w[4 * lane]), ll_value(w[4 * lane + 1]),
                                                       ll_value(w[4 * lane + 2]), ll_value(w[4 * lane + 3]));
                const float wgt = exp_cw(ms - mm);
                lsum = __fmaf_rn(ls, wgt, lsum);
                acc.x = __fmaf_rn(ov.x, wgt, acc.x);
                acc.y = __fmaf_rn(ov.y, wgt, acc.y);
                acc.z = __fmaf_rn(ov.z, wgt, acc.z);
                acc.w = __fmaf_rn(ov.w, wgt, acc.w);
            }
            const float inv = __fdiv_rn(1.0f, lsum);
            result = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
        }
    } else if (head_warp) {
        // More splits than the staging area holds: poll them in turn.
        result = mk_merge_direct(part + warp * pstride, splits, groups * pstride, tag_part, mrun, l_run, o, lane, ok);
    }
    if (mk_stop(flags, !ok)) return false;
    if (l == 1) H4B_TRACE(1504);
    if (l == 2) H4B_TRACE_CTA(20);
    float mx = 0.f;
    if (head_warp) {
        unsigned long long* att = xw + a.x.att + static_cast<long long>(qh) * d + 4 * lane;
        ll_store2(att, result.x, result.y, tag_att);
        ll_store2(att + 2, result.z, result.w, tag_att);
        mx = warp_max(fmaxf(fmaxf(fabsf(result.x), fabsf(result.y)), fmaxf(fabsf(result.z), fabsf(result.w))));
    }
    if (lane == 0) red[warp] = head_warp ? mx : 0.f;
    named_sync(1, kMkConsumers);
    if (threadIdx.x == 0) {
        float t = red[0];
        for (int w = 1; w < kMkWarps; ++w) t = fmaxf(t, red[w]);
        ll_store(xw + a.x.att_max + h, t, tag_att);
    }
    named_sync(1, kMkConsumers);  // red is reused by the next phase
    if (l == 1) H4B_TRACE(1505);
    if (l == 2) H4B_TRACE_CTA(21);
    return true;
}

struct MkSmem {
    int bars, red, geo, xq, gamma, consts, acc, scale, xo, att, ring, total;
};

__host__ __device__ inline MkSmem mk_smem_layout(int xq_bytes, int hidden, int rows_cap, int kv_bytes, int stages,
                                                 int slot_bytes) {
    MkSmem s;
    s.bars = 0;
    s.red = 2 * kMkMaxStages * 8;
    s.geo = s.red + 64 * 4;
    s.xq = s.geo + 128;  // kSegKinds SegGeo entries
    s.gamma = s.xq + xq_region(xq_bytes);
    s.consts = s.gamma + ((hidden * 4 + 127) & ~127);  // attention's q/k norm weights + RoPE row
    s.acc = s.consts + (3 + kMaxGroups) * kHeadDim * 4;  // + one staged q head per warp
    s.scale = s.acc + rows_cap * 4;    // two buffers: this phase's row scales and the next one's
    s.xo = s.scale + 2 * rows_cap * 4;  // this CTA's rows of x, kept across phases
    s.att = (s.xo + rows_cap * 4 + 127) & ~127;
    const int att_bytes = 2 * kSubTile * (kHeadDim + 16 / kv_bytes) * kv_bytes;
    s.ring = (s.att + (att_bytes > hidden * 4 ? att_bytes : hidden * 4) + 127) & ~127;
    s.total = s.ring + stages * slot_bytes + 512;  // slot loads may run up to 496 B past a tile
    return s;
}

// LM-head epilogue: logits, this CTA's greedy key as two exchange words,
// then CTA 0 takes the max over every CTA's key and writes the step's token
// and position (cpu_lightspark.py:704-705).
__device__ void mk_finish_token(const MkArgs& a, const Seg& sg, const float* sc_s, float act, int32_t* acc_s,
                                unsigned long long* xw, uint32_t tag_final, int pos, int* flags) {
    const h4b_state& st = a.s;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int cta = blockIdx.x, nctas = gridDim.x;
    unsigned long long best = 0ull;
    #pragma unroll 1
    for (int i = tid; i < sg.nrows; i += kMkConsumers) {
        const float v = mk_value(acc_s, sc_s, i, act);
        __stcg(st.logits + sg.r0 + i, v);
        const unsigned long long k = argmax_key(v, static_cast<uint32_t>(sg.r0 + i));
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    unsigned long long* keys = reinterpret_cast<unsigned long long*>(acc_s);
    named_sync(1, kMkConsumers);
    if (lane == 0) keys[warp] = best;
    named_sync(1, kMkConsumers);
    if (tid == 0) {
        for (int w = 0; w < kMkWarps; ++w) best = keys[w] > best ? keys[w] : best;
        ll_store_raw2(xw + a.x.keys + 2 * cta, (static_cast<unsigned long long>(tag_final) << 32) | (best >> 32),
                      (static_cast<unsigned long long>(tag_final) << 32) | (best & 0xFFFFFFFFull));
    }
    if (cta != 0) return;
    named_sync(1, kMkConsumers);
    bool failed = false;
    best = 0ull;
    #pragma unroll 1
    for (int c = tid; c < nctas; c += kMkConsumers) {
        const unsigned long long* p = xw + a.x.keys + 2 * c;
        PollClock clk;
        ulonglong2 w = ll_load2(p);
        while (ll_tag(w.x) != tag_final || ll_tag(w.y) != tag_final) {
            if (poll_expired(clk)) {
                failed = true;
                break;
            }
            w = ll_load2(p);
        }
        const unsigned long long k = ((w.x & 0xFFFFFFFFull) << 32) | (w.y & 0xFFFFFFFFull);
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    if (lane == 0) keys[warp] = best;
    if (mk_stop(flags, failed)) return;
    if (tid == 0) {
        for (int w = 0; w < kMkWarps; ++w) best = keys[w] > best ? keys[w] : best;
        *st.argmax_key = best;
        const int32_t id = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(best & 0xFFFFFFFFull));
        *st.next_token = id;
        *st.token = id;
        *st.position = pos + 1;
    }
}

template <typename KV>
__global__ void __launch_bounds__(kMkThreads, 1) decode_persistent_kernel(const MkArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const h4b_model& m = a.m;
    const h4b_state& st = a.s;
    const MkSmem L = mk_smem_layout(a.xq_bytes, m.hidden, a.rows_cap, sizeof(KV), a.stages, a.slot_bytes);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
    uint64_t* empty = full + kMkMaxStages;
    float* red = reinterpret_cast<float*>(smem + L.red);
    int* flags = reinterpret_cast<int*>(red + 32);  // [0] stop request, [1] consumers' snapshot, [2] tag base
    SegGeo* geo = reinterpret_cast<SegGeo*>(smem + L.geo);
    int8_t* xq = reinterpret_cast<int8_t*>(smem + L.xq);
    float* gamma_s = reinterpret_cast<float*>(smem + L.gamma);
    int32_t* acc_s = reinterpret_cast<int32_t*>(smem + L.acc);
    float* sc_base = reinterpret_cast<float*>(smem + L.scale);
    float* consts_s = reinterpret_cast<float*>(smem + L.consts);
    float* xo = reinterpret_cast<float*>(smem + L.xo);
    KV* ks = reinterpret_cast<KV*>(smem + L.att);
    KV* vs = ks + kSubTile * kv_row_stride<KV>();
    float* xs = reinterpret_cast<float*>(smem + L.att);  // embedding row, before any attention
    uint8_t* ring = smem + L.ring;
    unsigned long long* xw = st.exchange;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int cta = blockIdx.x, nctas = gridDim.x;
    const int L_layers = m.layers, H = m.hidden;
    const int pos = *st.position;
    const int token = *st.token;
    H4B_TRACE(0);

    if (tid == 0) {
        // This CTA's launch counter advances on every launch, whatever happens
        // later, so the tags of all CTAs stay in step.
        unsigned long long* gen = xw + a.x.gen + cta;
        const uint32_t g = static_cast<uint32_t>(*gen);
        *gen = g + 1u;
        flags[2] = static_cast<int>(mk_tag_base(g, L_layers));
        for (int s = 0; s < a.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);  // released by the owning consumer warp
        }
        flags[0] = wait_failed_before() ? 1 : 0;
        flags[1] = 0;
        if (pos < 0 || pos >= st.capacity) {
            if (cta == 0) report(kStatusBadPosition);
            flags[0] = 1;
        }
        fence_mbar_init();
    }
    if (warp == 1 && lane == 0) mk_geometry(a, cta, nctas, geo);
    __syncthreads();
    if (flags[0]) return;  // before any bulk copy is issued
    const uint32_t tbase = static_cast<uint32_t>(flags[2]);

    if (warp == kMkWarps) {
        // ---------------- producer warp: the whole token's weights ----------------
        if (lane == 0) {
            uint32_t seq = 0;
            bool stop = false;
            for (int g = 0; g <= 4 * L_layers && !stop; ++g) {
                const Seg sg = mk_segment(a, geo, g);
                for (int t = 0; t < sg.ntiles; ++t, ++seq) {
                    const int slot = seq % a.stages;
                    if (seq >= static_cast<uint32_t>(a.stages)) {
                        if (!mbar_wait(&empty[slot], ((seq / a.stages) - 1) & 1) ||
                            *reinterpret_cast<volatile int*>(&flags[0])) {
                            atomicOr(&flags[0], 1);
                            stop = true;
                            break;
                        }
                    }
                    const int rows_t = min(sg.tile_rows, sg.nrows - t * sg.tile_rows);
                    const uint32_t bytes = static_cast<uint32_t>(rows_t) * sg.kb;
                    if (seq >= 40 && seq < 140) H4B_TRACE_ANY(1400 + seq - 40);
                    mbar_arrive_expect_tx(&full[slot], bytes);
                    bulk_g2s(ring + static_cast<size_t>(slot) * a.slot_bytes,
                             sg.w + static_cast<size_t>(sg.r0 + t * sg.tile_rows) * sg.kb, bytes, &full[slot]);
                }
            }
            // Never leave the CTA with bulk copies in flight.
            const uint32_t first = seq > static_cast<uint32_t>(a.stages) ? seq - a.stages : 0;
            for (uint32_t t = first; t < seq; ++t) mbar_wait(&full[t % a.stages], (t / a.stages) & 1, 100000000ull);
        }
        __syncwarp();
        return;
    }

    // ---------------- consumer warps ----------------
    // One pass per GEMV segment g (per layer: qkv, o, gate/up, down; then the
    // LM head): prologue (RMSNorm or quantisation of the polled input), this
    // segment's ring tiles, epilogue. Each routine has one call site.
    uint32_t seq = 0;
    const float eps = m.eps;
    // Embedding (cpu_lightspark.py:341-349), computed by every CTA into xs;
    // the rows this CTA owns in the o/down partition start its copy of x.
    {
        const Seg so = mk_segment(a, geo, SEG_O);
        const bool ok = token >= 0 && token < m.vocab;
        if (!ok && cta == 0 && tid == 0) report(kStatusBadToken);
        const float scale = ok ? m.s_embed[token] : 0.f;
        const uint8_t* row = m.w_embed + static_cast<size_t>(ok ? token : 0) * (H >> 1);
        #pragma unroll 1
        for (int j = tid; j < (H >> 1); j += kMkConsumers) {
            const int8_t byte = static_cast<int8_t>(row[j]);
            xs[2 * j] = ok ? __fmul_rn(static_cast<float>(static_cast<int8_t>(byte << 4) >> 4), scale) : 0.f;
            xs[2 * j + 1] = ok ? __fmul_rn(static_cast<float>(byte >> 4), scale) : 0.f;
        }
        named_sync(1, kMkConsumers);
        #pragma unroll 1
        for (int i = tid; i < so.nrows; i += kMkConsumers) xo[i] = xs[so.r0 + i];
    }

    const int ctx = pos + 1;
    const int splits = max(1, min(a.max_splits, (ctx + a.attn_chunk - 1) / a.attn_chunk));
    const int items = m.kv_heads * splits;
    const int last = 4 * L_layers;

    for (int g = 0; g <= last; ++g) {
        const int l = g >> 2;
        const int kind = g == last ? 4 : (g & 3);  // SEG_* or 4 = LM head
        const uint32_t tl = tbase + kTagsPerLayer * l;
        const Seg sg = mk_segment(a, geo, g);
        const float* sc_s = sc_base + (g & 1) * a.rows_cap;
        H4B_TRACE(8 + 3 * g);
        if (g >= 8 && g < 12) H4B_TRACE_CTA(4 * (g - 8));
        if (g == last) H4B_TRACE_CTA(23);  // the LM head segment
#ifdef H4B_PHASE_TRACE
        if (g >= 8 && g < 12 && threadIdx.x == 0) {
            // one L2 round trip of a word that is already there (this CTA's own launch counter)
            const uint64_t t0 = globaltimer_ns();
            const unsigned long long w = ll_load(xw + a.x.gen + cta);
            uint64_t t1;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1) : "l"(w));  // waits for w
            H4B_TRACE_VAL(1650 + (g - 8), t1 - t0);
        }
#endif
        mk_fetch_own(a, g, geo, sc_base, gamma_s);
        async_copy_commit();  // group: this segment's scales and norm weight
        if (kind == SEG_QKV && l > 0 && cta < items)  // layer 0: xs still holds the embedding
            mk_attention_fetch<KV>(a, l, cta / splits, cta % splits, splits, pos, ks, vs, consts_s);
        async_copy_commit();  // group: attention's first K/V sub-tile (empty elsewhere)

        // ---- prologue ----
        float act;
        if (kind == SEG_O || kind == SEG_DOWN) {
            const bool o = kind == SEG_O;
            act = mk_prologue_quant(xw + (o ? a.x.att : a.x.act), xw + (o ? a.x.att_max : a.x.act_max),
                                    o ? m.kv_heads : nctas, tl + (o ? TAG_ATT : TAG_ACT),
                                    o ? m.heads * m.head_dim : m.intermediate, xq, red, flags,
                                    g >= 8 && g < 12 ? 1600 + 2 * (g - 8) : -1);
        } else {
            // qkv reads x after the previous layer's down (layer 0: the
            // embedding in xs), gate/up after this layer's o, the head after
            // the last down.
            const bool from_xs = g == 0;
            const unsigned long long* src = xw + (kind == SEG_GATE_UP ? a.x.x_o : a.x.x_down);
            const uint32_t tag = kind == SEG_GATE_UP ? tl + TAG_XO : tl - kTagsPerLayer + TAG_XDOWN;
            act = mk_prologue_rms(from_xs ? xs : nullptr, from_xs ? nullptr : src, tag, gamma_s, H, eps, xq, red,
                                  flags, g >= 8 && g < 12 ? 1600 + 2 * (g - 8) : -1);
        }
        H4B_TRACE(8 + 3 * g + 1);
        if (g >= 8 && g < 12) H4B_TRACE_CTA(4 * (g - 8) + 1);
        if (g == last) H4B_TRACE_CTA(24);  // the LM head segment
        if (g >= 8 && g < 12) H4B_TRACE(1700 + (g - 8));

        // ---- tiles ----
        mk_run_tiles(sg, seq, a.stages, a.slot_bytes, ring, full, empty, xq, acc_s, flags,
                     g >= 8 && g < 12 ? 1710 + (g - 8) : -1);
        seq += sg.ntiles;
        H4B_TRACE(8 + 3 * g + 2);
        if (g >= 8 && g < 12) H4B_TRACE_CTA(4 * (g - 8) + 2);
        if (g == last) H4B_TRACE_CTA(25);  // the LM head segment
        if (mk_stop(flags)) return;

        // ---- epilogue ----
        if (kind == SEG_QKV) {
            #pragma unroll 1
            for (int i = tid; i < sg.nrows; i += kMkConsumers)
                ll_store(xw + a.x.qkv + sg.r0 + i, mk_value(acc_s, sc_s, i, act), tl + TAG_QKV);
            if (cta < items &&
                !mk_attention<KV>(a, xw, tbase, l, cta / splits, cta % splits, splits, pos, ks, vs, consts_s, red,
                                  flags, l > 0))
                return;
        } else if (kind == SEG_O || kind == SEG_DOWN) {
            const long long dst = kind == SEG_O ? a.x.x_o : a.x.x_down;
            const uint32_t tag = tl + (kind == SEG_O ? TAG_XO : TAG_XDOWN);
            #pragma unroll 1
            for (int i = tid; i < sg.nrows; i += kMkConsumers) {
                xo[i] = __fadd_rn(xo[i], mk_value(acc_s, sc_s, i, act));
                ll_store(xw + dst + sg.r0 + i, xo[i], tag);
            }
        } else if (kind == SEG_GATE_UP) {
            float local = 0.f;
            #pragma unroll 1
            for (int p = tid; p < (sg.nrows >> 1); p += kMkConsumers) {
                const int b = p / kSwigluBlock, j = p % kSwigluBlock;
                const int gi = 2 * kSwigluBlock * b + j;
                const float gte = mk_value(acc_s, sc_s, gi, act), u = mk_value(acc_s, sc_s, gi + kSwigluBlock, act);
                const float y = __fmul_rn(__fdiv_rn(gte, __fadd_rn(1.0f, exp_cw(-gte))), u);
                ll_store(xw + a.x.act + (sg.r0 >> 1) + p, y, tl + TAG_ACT);
                local = fmaxf(local, fabsf(y));
            }
            const float mx = group_max(local, red, kMkWarps, 1);
            if (tid == 0) ll_store(xw + a.x.act_max + cta, mx, tl + TAG_ACT);
        } else {
            mk_finish_token(a, sg, sc_s, act, acc_s, xw, tl, pos, flags);
        }
        if (g >= 8 && g < 12) H4B_TRACE_CTA(4 * (g - 8) + 3);
        if (g == last) H4B_TRACE_CTA(26);  // the LM head segment
    }
}

struct MkPlan {
    MkArgs args;
    int smem;
};

int mk_splits_max(const h4b_model* m) {
    return std::max(1, std::min(64, sm_count() / m->kv_heads));
}

// Tuning builds (-DH4B_TUNING) read overrides of the plan's knobs from the
// environment; the normal build uses the defaults.
static int tuning_env(const char* name, int fallback) {
#ifdef H4B_TUNING
    const char* e = std::getenv(name);  // read per plan: a captured graph keeps its value
    if (e && *e) return std::max(1, std::atoi(e));
#else
    (void)name;
#endif
    return fallback;
}

static int plan_persistent(const h4b_model* m, const h4b_state* s, MkPlan* p) {
    int rc = validate(m, s);
    if (rc) return rc;
    if (!s->exchange || (reinterpret_cast<uintptr_t>(s->exchange) & 15)) return H4B_EINVAL;
    if (m->hidden > kMkMaxHidden || m->hidden % 8 || m->intermediate % 8) return H4B_EUNSUPPORTED;
    const int q_size = m->heads * m->head_dim;
    const int max_width = std::max(m->hidden, std::max(q_size, m->intermediate));
    if (max_width > kMkMaxWidth) return H4B_EUNSUPPORTED;
    const int nctas = sm_count();
    if (nctas > kMkConsumers || nctas > kMkMaxCtas) return H4B_EUNSUPPORTED;  // one act maximum per thread
    if (static_cast<long long>(std::max(m->vocab, 2 * m->intermediate)) * nctas >= (1ll << 32))
        return H4B_EUNSUPPORTED;  // mk_geometry's 32-bit row partition
    if (std::max(q_size, m->intermediate) > kMkQuantGroups * 8 * kMkConsumers) return H4B_EUNSUPPORTED;
    if (m->heads / m->kv_heads > kMkWarps) return H4B_EUNSUPPORTED;  // one consumer warp per q head of a group
    MkArgs& a = p->args;
    a = MkArgs{};
    a.m = *m;
    a.s = *s;
    a.x = x_layout(*m);
    a.attn_chunk = tuning_env("H4B_ATTN_CHUNK", 32);
    a.max_splits = mk_splits_max(m);
    {
        const int groups = m->heads / m->kv_heads;
        const int kvb = s->kv_dtype == 0 ? 4 : 2;
        const int staging = 2 * kSubTile * (kHeadDim + 16 / kvb) * kvb;
        a.stage_splits = staging / (groups * kPartialStride * 8);
    }
    a.xq_bytes = max_width;
    // Rows one CTA owns in any segment, plus one partition unit of slack.
    const int biggest = std::max({m->vocab, 2 * m->intermediate, q_size + 2 * m->kv_heads * m->head_dim, m->hidden});
    a.rows_cap = ((biggest + nctas - 1) / nctas + 2 * kSwigluBlock + 31) & ~31;
    const int kv_bytes = s->kv_dtype == 0 ? 4 : 2;
    const MkSmem base = mk_smem_layout(a.xq_bytes, m->hidden, a.rows_cap, kv_bytes, 0, 0);
    const int budget = 227 * 1024 - base.total;
    a.stages = kMkStages;
    a.slot_bytes = std::min(kMkMaxSlotBytes, budget / kMkStages / 1024 * 1024);
    if (a.slot_bytes < max_width / 2) return H4B_EUNSUPPORTED;  // one row must fit a slot
    p->smem = mk_smem_layout(a.xq_bytes, m->hidden, a.rows_cap, kv_bytes, a.stages, a.slot_bytes).total;
    return 0;
}

int prepare_persistent() {
    H4B_CUDA_TRY(cudaFuncSetAttribute(decode_persistent_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      227 * 1024));
    H4B_CUDA_TRY(cudaFuncSetAttribute(decode_persistent_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      227 * 1024));
    return 0;
}

int decode_persistent(const h4b_model* m, const h4b_state* s, cudaStream_t stream) {
    {
        const int prc = prepare_kernels();
        if (prc) return prc;
    }
    MkPlan p;
    int rc = plan_persistent(m, s, &p);
    if (rc) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sm_count());
    cfg.blockDim = dim3(kMkThreads);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (s->kv_dtype == 0) H4B_CUDA_TRY(cudaLaunchKernelEx(&cfg, decode_persistent_kernel<float>, p.args));
    else H4B_CUDA_TRY(cudaLaunchKernelEx(&cfg, decode_persistent_kernel<__half>, p.args));
    return 0;
}

}  // namespace h4b

#ifdef H4B_PHASE_TRACE
// Copies the phase timeline (3 x 2048 u64) of the last traced launch to host.
extern "C" int h4b_phase_trace(unsigned long long* host) {
    H4B_CUDA_TRY(cudaDeviceSynchronize());
    H4B_CUDA_TRY(cudaMemcpyFromSymbol(host, h4b::g_phase_trace, sizeof(unsigned long long) * 3 * 2048));
    return 0;
}

extern "C" int h4b_phase_trace_ctas(unsigned long long* host) {
    H4B_CUDA_TRY(cudaDeviceSynchronize());
    H4B_CUDA_TRY(cudaMemcpyFromSymbol(host, h4b::g_phase_all, sizeof(unsigned long long) * 1024 * 16));
    return 0;
}
#endif

extern "C" int h4b_decode_persistent(const h4b_model* model, const h4b_state* state, void* stream) {
    return h4b::decode_persistent(model, state, static_cast<cudaStream_t>(stream));
}

extern "C" long long h4b_persistent_exchange_words(const h4b_model* model) {
    if (!model || model->layers < 1 || model->kv_heads < 1 || model->heads % model->kv_heads) return H4B_EINVAL;
    return h4b::x_layout(*model).total;
}
