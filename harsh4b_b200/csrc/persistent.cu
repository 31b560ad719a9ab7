// Persistent decode step: one cooperative kernel per token, one CTA per SM.
//
// Same arithmetic as the kernel chain in decode.cu (the same prologues,
// tile math, epilogues and attention order), organised so the weight stream
// never stops at a phase boundary:
//
//   * the producer warp of each CTA walks that SM's rows of every weight
//     matrix of the token in phase order (per layer qkv, o, gate/up, down;
//     then the LM head) and streams them through one shared-memory ring of
//     8 KB slots with 1-D bulk copies, waiting only for free slots;
//   * the eight consumer warps run the phases: wait for the phase's input
//     (a release/acquire counter that every producing CTA bumps once),
//     quantise the input (prologue), consume this phase's ring tiles, write
//     the outputs (epilogue) and bump the phase counter;
//   * attention runs on the first kv_heads * S CTAs (S chosen per token from
//     the context length); the last CTA of each kv head merges the splits.
//
// The ring covers a few microseconds of this SM's share of HBM bandwidth,
// so the producer keeps loading the next phases' weights while consumers
// wait on a dependency. Every wait is bounded; a CTA that gives up sets the
// status word and every other CTA then stops at its next wait.
#include "common.cuh"

namespace h4b {

constexpr int kMkWarps = 8;  // consumer warps
constexpr int kMkConsumers = kMkWarps * 32;
constexpr int kMkThreads = kMkConsumers + 32;
constexpr int kMkMaxSlotBytes = 16384;
constexpr int kMkStages = 16;  // a multiple of kMkWarps: each ring slot has one owning warp
constexpr int kMkMaxStages = kMkStages;
constexpr int kMkMaxHidden = 8192;  // RMSNorm inputs kept in registers (4 groups of 8 per thread)
constexpr int kMkMaxWidth = 16384;

enum { SEG_QKV = 0, SEG_O = 1, SEG_GATE_UP = 2, SEG_DOWN = 3 };

struct MkArgs {
    h4b_model m;
    h4b_state s;
    uint32_t* ready;       // [5 * layers + 2] phase counters
    uint32_t* attn_count;  // [layers][kv_heads] split-merge counters
    int stages;
    int slot_bytes;        // ring slot size (a tile is at most one slot)
    int attn_chunk;        // target tokens per attention split
    int max_splits;        // splits per kv head at most
    int xq_bytes, rows_cap;
};

// Phase counter indices.
__host__ __device__ inline int ph_qkv(int l) { return 5 * l; }
__host__ __device__ inline int ph_attn(int l) { return 5 * l + 1; }
__host__ __device__ inline int ph_o(int l) { return 5 * l + 2; }
__host__ __device__ inline int ph_gate_up(int l) { return 5 * l + 3; }
__host__ __device__ inline int ph_down(int l) { return 5 * l + 4; }

struct Seg {
    const uint8_t* w;
    const float* ws;
    int width, kb, r0, nrows, tile_rows, ntiles;
};

// Rows of GEMV segment g (4 per layer, then the LM head) that CTA `cta` owns.
__device__ __forceinline__ Seg mk_segment(const MkArgs& a, int g, int cta, int nctas) {
    const h4b_model& m = a.m;
    const int H = m.hidden, I = m.intermediate;
    const int Q = m.heads * m.head_dim, KV = m.kv_heads * m.head_dim;
    Seg s;
    int rows, align = 1;
    if (g == 4 * m.layers) {
        s.w = m.w_embed; s.ws = m.s_embed; rows = m.vocab; s.width = H;
    } else {
        const int l = g >> 2;
        switch (g & 3) {
            case SEG_QKV:
                rows = Q + 2 * KV; s.width = H;
                s.w = m.w_qkv + static_cast<size_t>(l) * rows * (H / 2);
                s.ws = m.s_qkv + static_cast<size_t>(l) * rows;
                break;
            case SEG_O:
                rows = H; s.width = Q;
                s.w = m.w_o + static_cast<size_t>(l) * H * (Q / 2);
                s.ws = m.s_o + static_cast<size_t>(l) * H;
                break;
            case SEG_GATE_UP:
                rows = 2 * I; s.width = H; align = 2 * kSwigluBlock;
                s.w = m.w_gate_up + static_cast<size_t>(l) * 2 * I * (H / 2);
                s.ws = m.s_gate_up + static_cast<size_t>(l) * 2 * I;
                break;
            default:
                rows = H; s.width = I;
                s.w = m.w_down + static_cast<size_t>(l) * H * (I / 2);
                s.ws = m.s_down + static_cast<size_t>(l) * H;
                break;
        }
    }
    s.kb = s.width >> 1;
    const int units = rows / align;
    const int u0 = static_cast<int>(static_cast<long long>(cta) * units / nctas);
    const int u1 = static_cast<int>(static_cast<long long>(cta + 1) * units / nctas);
    s.r0 = u0 * align;
    s.nrows = (u1 - u0) * align;
    s.tile_rows = max(1, min((s.nrows + kMkWarps - 1) / kMkWarps, a.slot_bytes / s.kb));
    s.ntiles = (s.nrows + s.tile_rows - 1) / s.tile_rows;
    return s;
}

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// The consumers' stop decision. flags[0] is a stop request any warp may set
// at any time (the producer included); flags[1] is a snapshot only consumer
// thread 0 writes, before named barrier 1, and every consumer reads after
// it -- so all consumer threads take the same branch and none is left
// waiting at a later named barrier.
__device__ bool mk_stop(int* flags, bool own_failure = false) {
    if (threadIdx.x == 0) {
        if (own_failure) atomicOr(&flags[0], 1);
        flags[1] = *reinterpret_cast<volatile int*>(&flags[0]);
    }
    named_sync(1, kMkConsumers);
    return flags[1] != 0;
}

// Consumer-side dependency wait: thread 0 polls; returns false (for every
// consumer thread alike) if the CTA must stop.
__device__ bool mk_wait(const uint32_t* counter, uint32_t target, int* flags) {
    bool failed = false;
    if (threadIdx.x == 0 && ld_acquire_u32(counter) < target) {
        const uint64_t start = globaltimer_ns();
        for (uint32_t spin = 1; ld_acquire_u32(counter) < target; ++spin) {
            __nanosleep(32);  // keep the poll off the issue slots of the working warps
            if ((spin & 63) != 0) continue;
            if (wait_failed_before() || *reinterpret_cast<volatile int*>(&flags[0])) {
                failed = true;
                break;
            }
            if (globaltimer_ns() - start > kWaitLimitNs) {
                report(kStatusWaitTimeout);
                failed = true;
                break;
            }
        }
    }
    return !mk_stop(flags, failed);
}

// All consumer writes of this phase are done: publish them.
__device__ __forceinline__ void mk_signal(uint32_t* counter) {
    named_sync(1, kMkConsumers);
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(counter, 1u);
    }
}

__device__ __forceinline__ void load8_cg(const float* p, float v[8]) {
    const float4 a = __ldcg(reinterpret_cast<const float4*>(p));
    const float4 b = __ldcg(reinterpret_cast<const float4*>(p + 4));
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// RMSNorm + absmax quantisation of x (n <= kMkMaxHidden) into xq, in the
// same order as the GEMV kernel's prologue; returns the dequant scale.
__device__ float mk_prologue_rms(const float* x, bool from_smem, const float* gamma_s, int n, float eps,
                                 int8_t* xq, float* red) {
    const int tid = threadIdx.x;
    const int groups = n >> 3;
    float v[4][8];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int g = tid + k * kMkConsumers;
        if (g < groups) {
            if (from_smem) load8(x + 8 * g, v[k]);
            else load8_cg(x + 8 * g, v[k]);
#pragma unroll
            for (int e = 0; e < 8; ++e) ss = __fmaf_rn(v[k][e], v[k][e], ss);
        }
    }
    ss = group_sum(ss, red, kMkWarps, 1);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(n)), eps)));
    float local = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int g = tid + k * kMkConsumers;
        if (g < groups) {
            float gm[8];
            load8(gamma_s + 8 * g, gm);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                v[k][e] = __fmul_rn(__fmul_rn(v[k][e], inv), gm[e]);
                local = fmaxf(local, fabsf(v[k][e]));
            }
        }
    }
    const float m = group_max(local, red, kMkWarps, 1);
    const float qs = quant_multiplier(m);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int g = tid + k * kMkConsumers;
        if (g < groups) {
            int q[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) q[e] = quantize_one(v[k][e], qs);
            store_group(xq, g, q);
        }
    }
    zero_xq_tail(xq, n, tid, kMkConsumers);
    named_sync(1, kMkConsumers);
    return dequant_scale(m);
}

// Quantisation of v with the absmax its producers published.
__device__ float mk_prologue_quant(const float* v, const float* absmax_slot, int n, int8_t* xq) {
    const float m = __ldcg(absmax_slot);
    const float qs = quant_multiplier(m);
    for (int g = threadIdx.x; g < (n >> 3); g += kMkConsumers) {
        float x[8];
        int q[8];
        load8_cg(v + 8 * g, x);
#pragma unroll
        for (int e = 0; e < 8; ++e) q[e] = quantize_one(x[e], qs);
        store_group(xq, g, q);
    }
    zero_xq_tail(xq, n, threadIdx.x, kMkConsumers);
    named_sync(1, kMkConsumers);
    return dequant_scale(m);
}

// This CTA's tiles of one GEMV segment: int32 row sums into acc_s.
template <int SLOTS, int RB>
__device__ void mk_tiles(const Seg& sg, uint32_t seq0, int stages, int slot_bytes, const uint8_t* ring, uint64_t* full,
                         uint64_t* empty, const int8_t* xq, int32_t* acc_s, int* flags) {
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
    for (int t = warp; t < sg.ntiles; t += kMkWarps) {
        const uint32_t gseq = seq0 + t;
        const int slot = gseq % stages;
        if (*reinterpret_cast<volatile int*>(&flags[0])) break;
        if (!mbar_wait(&full[slot], (gseq / stages) & 1)) {
            atomicOr(&flags[0], 1);
            break;
        }
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
    }
    named_sync(1, kMkConsumers);  // acc_s complete
}

__device__ void mk_run_tiles(const Seg& sg, uint32_t seq0, int stages, int slot_bytes, const uint8_t* ring, uint64_t* full,
                             uint64_t* empty, const int8_t* xq, int32_t* acc_s, int* flags) {
    const int need = ((sg.width >> 5) + 31) / 32;
    if (need <= 1) mk_tiles<1, 2>(sg, seq0, stages, slot_bytes, ring, full, empty, xq, acc_s, flags);
    else if (need <= 2) mk_tiles<2, 2>(sg, seq0, stages, slot_bytes, ring, full, empty, xq, acc_s, flags);
    else if (need <= 3) mk_tiles<3, 2>(sg, seq0, stages, slot_bytes, ring, full, empty, xq, acc_s, flags);
    else if (need <= 4) mk_tiles<4, 2>(sg, seq0, stages, slot_bytes, ring, full, empty, xq, acc_s, flags);
    else if (need <= 6) mk_tiles<6, 2>(sg, seq0, stages, slot_bytes, ring, full, empty, xq, acc_s, flags);
    else if (need <= 8) mk_tiles<8, 2>(sg, seq0, stages, slot_bytes, ring, full, empty, xq, acc_s, flags);
    else if (need <= 10) mk_tiles<10, 2>(sg, seq0, stages, slot_bytes, ring, full, empty, xq, acc_s, flags);
    else if (need <= 12) mk_tiles<12, 2>(sg, seq0, stages, slot_bytes, ring, full, empty, xq, acc_s, flags);
    else mk_tiles<16, 2>(sg, seq0, stages, slot_bytes, ring, full, empty, xq, acc_s, flags);
}

// Starts the 4-byte async copies of a segment's row scales into sc_s.
__device__ __forceinline__ void mk_fetch_scales(const Seg& sg, float* sc_s) {
    for (int i = threadIdx.x; i < sg.nrows; i += kMkConsumers) async_copy4(sc_s + i, sg.ws + sg.r0 + i);
}

// Starts the async copy of an RMSNorm weight (n floats) into gamma_s.
__device__ __forceinline__ void mk_fetch_gamma(const float* gamma, float* gamma_s, int n) {
    for (int i = threadIdx.x; i < n; i += kMkConsumers) async_copy4(gamma_s + i, gamma + i);
}

__device__ __forceinline__ float mk_value(const int32_t* acc_s, const float* sc_s, int i, float act_scale) {
    return __fmul_rn(__fmul_rn(static_cast<float>(acc_s[i]), act_scale), sc_s[i]);
}

// One attention split (kv head h, split `split` of `splits`) for layer l,
// in the order of gqa_split_kernel; the last split of head h merges.
template <typename KV>
__device__ void mk_attention(const MkArgs& a, int l, int h, int split, int splits, int pos, KV* ks, KV* vs,
                             float* red, int* flags) {
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
    const float* cs = m.rope_cos + static_cast<long long>(pos) * (d / 2);
    const float* sn = m.rope_sin + static_cast<long long>(pos) * (d / 2);
    const float* qn = m.norm_q + static_cast<size_t>(l) * d;
    const float* kn = m.norm_k + static_cast<size_t>(l) * d;
    const size_t kv_layer = static_cast<size_t>(m.kv_heads) * st.capacity * d;
    KV* kc = static_cast<KV*>(st.k_cache) + l * kv_layer + static_cast<size_t>(h) * st.capacity * d;
    KV* vc = static_cast<KV*>(st.v_cache) + l * kv_layer + static_cast<size_t>(h) * st.capacity * d;

    float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
    if (head_warp) {
        q = __ldcg(reinterpret_cast<const float4*>(st.qkv + static_cast<long long>(qh) * d + 4 * lane));
        q = norm_rope(q, qn, cs, sn, m.eps, lane);
    }
    const bool owns_new = t0 <= pos && pos < t1;
    float4 k_new = make_float4(0.f, 0.f, 0.f, 0.f), v_new = k_new;
    if (owns_new) {
        if (warp == 0) {
            k_new = __ldcg(reinterpret_cast<const float4*>(st.qkv + q_size + static_cast<long long>(h) * d + 4 * lane));
            k_new = norm_rope(k_new, kn, cs, sn, m.eps, lane);
            store4<KV>(kc + static_cast<long long>(pos) * d + 4 * lane, k_new);
        }
        if (warp == groups - 1) {
            v_new = __ldcg(reinterpret_cast<const float4*>(st.qkv + q_size + kv_size + static_cast<long long>(h) * d +
                                                            4 * lane));
            store4<KV>(vc + static_cast<long long>(pos) * d + 4 * lane, v_new);
        }
    }
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(d)));
    constexpr int kRowVecs = kHeadDim * sizeof(KV) / 16;
    float mrun = -INFINITY, l_run = 0.f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int base = t0; base < t1; base += kSubTile) {
        const int n = min(kSubTile, t1 - base);
        named_sync(1, kMkConsumers);
        for (int i = threadIdx.x; i < 2 * n * kRowVecs; i += kMkConsumers) {
            const int which = i / (n * kRowVecs), rest = i % (n * kRowVecs);
            const int r = rest / kRowVecs, piece = rest % kRowVecs;
            if (base + r == pos && owns_new) continue;
            const KV* src = (which ? vc : kc) + static_cast<long long>(base + r) * d;
            reinterpret_cast<uint4*>((which ? vs : ks) + r * kHeadDim)[piece] =
                __ldcg(reinterpret_cast<const uint4*>(src) + piece);
        }
        if (owns_new && pos >= base && pos < base + n) {
            if (warp == 0) store4<KV>(ks + (pos - base) * kHeadDim + 4 * lane, k_new);
            if (warp == groups - 1) store4<KV>(vs + (pos - base) * kHeadDim + 4 * lane, v_new);
        }
        named_sync(1, kMkConsumers);
        if (head_warp) {
            float p_round[2];
            float mt = -INFINITY;
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                if (32 * r >= n) {
                    p_round[r] = -INFINITY;
                    continue;
                }
                float part[32];
#pragma unroll
                for (int t = 0; t < 32; ++t) {
                    const int tt = min(32 * r + t, n - 1);
                    part[t] = dot4(q, load4<KV>(ks + tt * kHeadDim + 4 * lane));
                }
                const float sc = __fmul_rn(transpose_reduce32(part, lane), scale);
                p_round[r] = (32 * r + lane < n) ? sc : -INFINITY;
                mt = fmaxf(mt, p_round[r]);
            }
            mt = warp_max(mt);
#pragma unroll
            for (int r = 0; r < 2; ++r) p_round[r] = (32 * r + lane < n) ? exp_cw(p_round[r] - mt) : 0.f;
            const float lt = warp_sum(p_round[0] + p_round[1]);
            float4 ot = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int t = 0; t < n; ++t) {
                const float p = __shfl_sync(0xffffffffu, p_round[t >> 5], t & 31);
                const float4 v = load4<KV>(vs + t * kHeadDim + 4 * lane);
                ot.x = __fmaf_rn(p, v.x, ot.x);
                ot.y = __fmaf_rn(p, v.y, ot.y);
                ot.z = __fmaf_rn(p, v.z, ot.z);
                ot.w = __fmaf_rn(p, v.w, ot.w);
            }
            const float mn = fmaxf(mrun, mt);
            const float c_old = exp_cw(mrun - mn), c_new = exp_cw(mt - mn);
            l_run = __fmaf_rn(l_run, c_old, __fmul_rn(lt, c_new));
            o.x = __fmaf_rn(o.x, c_old, __fmul_rn(ot.x, c_new));
            o.y = __fmaf_rn(o.y, c_old, __fmul_rn(ot.y, c_new));
            o.z = __fmaf_rn(o.z, c_old, __fmul_rn(ot.z, c_new));
            o.w = __fmaf_rn(o.w, c_old, __fmul_rn(ot.w, c_new));
            mrun = mn;
        }
    }

    float4 result = make_float4(0.f, 0.f, 0.f, 0.f);
    bool merged = false;
    if (splits == 1) {
        if (head_warp) {
            const float inv = __fdiv_rn(1.0f, l_run);
            result = make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
        }
        merged = true;
    } else {
        const int stride = kPartialStride;
        float* base = st.attn_partials + static_cast<long long>(h) * a.max_splits * groups * stride;
        if (head_warp) {
            float* mine = base + (static_cast<long long>(split) * groups + warp) * stride;
            __stcg(reinterpret_cast<float4*>(mine + 4 * lane), o);
            if (lane == 0) {
                __stcg(mine + kHeadDim, mrun);
                __stcg(mine + kHeadDim + 1, l_run);
            }
        }
        named_sync(1, kMkConsumers);
        if (threadIdx.x == 0) {
            __threadfence();
            const uint32_t prev = atomicAdd(&a.attn_count[l * m.kv_heads + h], 1u);
            flags[3] = (prev == static_cast<uint32_t>(splits - 1));
        }
        named_sync(1, kMkConsumers);
        if (flags[3]) {
            __threadfence();
            if (head_warp) result = merge_splits(base + warp * stride, splits, groups * stride, lane);
            merged = true;
        }
    }
    if (!merged) return;
    float mx = 0.f;
    if (head_warp) {
        __stcg(reinterpret_cast<float4*>(st.attended + static_cast<long long>(qh) * d + 4 * lane), result);
        mx = warp_max(fmaxf(fmaxf(fabsf(result.x), fabsf(result.y)), fmaxf(fabsf(result.z), fabsf(result.w))));
    }
    if (lane == 0) red[warp] = head_warp ? mx : 0.f;
    named_sync(1, kMkConsumers);
    if (threadIdx.x == 0) {
        float t = red[0];
        for (int w = 1; w < kMkWarps; ++w) t = fmaxf(t, red[w]);
        atomic_max_nonneg(st.absmax + 2 * l, t);
    }
    mk_signal(&a.ready[ph_attn(l)]);
}

struct MkSmem {
    int bars, red, xq, gamma, acc, scale, att, ring, total;
};

__host__ __device__ inline MkSmem mk_smem_layout(int xq_bytes, int hidden, int rows_cap, int kv_bytes, int stages,
                                                 int slot_bytes) {
    MkSmem s;
    s.bars = 0;
    s.red = 2 * kMkMaxStages * 8;
    s.xq = s.red + 64 * 4;
    s.gamma = s.xq + xq_region(xq_bytes);
    s.acc = s.gamma + ((hidden * 4 + 127) & ~127);
    s.scale = s.acc + rows_cap * 4;
    s.att = (s.scale + rows_cap * 4 + 127) & ~127;
    const int att_bytes = 2 * kSubTile * kHeadDim * kv_bytes;
    s.ring = (s.att + (att_bytes > hidden * 4 ? att_bytes : hidden * 4) + 127) & ~127;
    s.total = s.ring + stages * slot_bytes + 512;  // slot loads may run up to 496 B past a tile
    return s;
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
    int* flags = reinterpret_cast<int*>(red + 32);  // [0] stop request, [1] consumers' snapshot, [3] last split
    int8_t* xq = reinterpret_cast<int8_t*>(smem + L.xq);
    float* gamma_s = reinterpret_cast<float*>(smem + L.gamma);
    int32_t* acc_s = reinterpret_cast<int32_t*>(smem + L.acc);
    float* sc_s = reinterpret_cast<float*>(smem + L.scale);
    KV* ks = reinterpret_cast<KV*>(smem + L.att);
    KV* vs = ks + kSubTile * kHeadDim;
    float* xs = reinterpret_cast<float*>(smem + L.att);  // embedding row, before any attention
    uint8_t* ring = smem + L.ring;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int cta = blockIdx.x, nctas = gridDim.x;
    const int L_layers = m.layers, H = m.hidden;
    const int pos = *st.position;
    const int token = *st.token;

    if (tid == 0) {
        for (int s = 0; s < a.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);  // released by the owning consumer warp
        }
        flags[0] = wait_failed_before() ? 1 : 0;
        flags[1] = 0;
        flags[3] = 0;
        if (pos < 0 || pos >= st.capacity) {
            if (cta == 0) report(kStatusBadPosition);
            flags[0] = 1;
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (flags[0]) return;  // before any bulk copy is issued

    if (warp == kMkWarps) {
        // ---------------- producer warp: the whole token's weights ----------------
        if (lane == 0) {
            uint32_t seq = 0;
            bool stop = false;
            for (int g = 0; g <= 4 * L_layers && !stop; ++g) {
                const Seg sg = mk_segment(a, g, cta, nctas);
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
    uint32_t seq = 0;
    const float eps = m.eps;
    // Embedding (cpu_lightspark.py:341-349), computed by every CTA; the rows
    // this CTA later updates (its o/down partition) also go to global x.
    {
        const bool ok = token >= 0 && token < m.vocab;
        if (!ok && cta == 0 && tid == 0) report(kStatusBadToken);
        const float scale = ok ? m.s_embed[token] : 0.f;
        const uint8_t* row = m.w_embed + static_cast<size_t>(ok ? token : 0) * (H >> 1);
        for (int j = tid; j < (H >> 1); j += kMkConsumers) {
            const int8_t byte = static_cast<int8_t>(row[j]);
            xs[2 * j] = ok ? __fmul_rn(static_cast<float>(static_cast<int8_t>(byte << 4) >> 4), scale) : 0.f;
            xs[2 * j + 1] = ok ? __fmul_rn(static_cast<float>(byte >> 4), scale) : 0.f;
        }
        mk_fetch_gamma(m.norm_in, gamma_s, H);
        named_sync(1, kMkConsumers);
        const Seg so = mk_segment(a, SEG_O, cta, nctas);
        for (int i = tid; i < so.nrows; i += kMkConsumers) __stcg(st.x + so.r0 + i, xs[so.r0 + i]);
    }

    const int kv_heads = m.kv_heads;
    const int ctx = pos + 1;
    const int splits = max(1, min(a.max_splits, (ctx + a.attn_chunk - 1) / a.attn_chunk));
    const int items = kv_heads * splits;

    for (int l = 0; l < L_layers; ++l) {
        // ---- qkv: RMSNorm(x) -> quantise -> GEMV ----
        Seg sg = mk_segment(a, 4 * l + SEG_QKV, cta, nctas);
        mk_fetch_scales(sg, sc_s);
        if (l > 0) {
            mk_fetch_gamma(m.norm_in + static_cast<size_t>(l) * H, gamma_s, H);
            if (!mk_wait(&a.ready[ph_down(l - 1)], nctas, flags)) return;
        }
        async_copy_wait_all();
        named_sync(1, kMkConsumers);
        float act = mk_prologue_rms(l == 0 ? xs : st.x, l == 0, gamma_s, H, eps, xq, red);
        mk_run_tiles(sg, seq, a.stages, a.slot_bytes, ring, full, empty, xq, acc_s, flags);
        seq += sg.ntiles;
        if (mk_stop(flags)) return;
        for (int i = tid; i < sg.nrows; i += kMkConsumers) __stcg(st.qkv + sg.r0 + i, mk_value(acc_s, sc_s, i, act));
        mk_signal(&a.ready[ph_qkv(l)]);

        // ---- attention ----
        if (!mk_wait(&a.ready[ph_qkv(l)], nctas, flags)) return;
        if (cta < items) mk_attention<KV>(a, l, cta / splits, cta % splits, splits, pos, ks, vs, red, flags);

        // ---- o: quantise(attended) -> GEMV -> residual ----
        sg = mk_segment(a, 4 * l + SEG_O, cta, nctas);
        mk_fetch_scales(sg, sc_s);
        if (!mk_wait(&a.ready[ph_attn(l)], kv_heads, flags)) return;
        async_copy_wait_all();
        act = mk_prologue_quant(st.attended, st.absmax + 2 * l, m.heads * m.head_dim, xq);
        mk_run_tiles(sg, seq, a.stages, a.slot_bytes, ring, full, empty, xq, acc_s, flags);
        seq += sg.ntiles;
        if (mk_stop(flags)) return;
        for (int i = tid; i < sg.nrows; i += kMkConsumers)
            __stcg(st.x + sg.r0 + i, __fadd_rn(__ldcg(st.x + sg.r0 + i), mk_value(acc_s, sc_s, i, act)));
        mk_signal(&a.ready[ph_o(l)]);

        // ---- gate/up: RMSNorm(x) -> quantise -> GEMV -> SwiGLU ----
        sg = mk_segment(a, 4 * l + SEG_GATE_UP, cta, nctas);
        mk_fetch_scales(sg, sc_s);
        mk_fetch_gamma(m.norm_post + static_cast<size_t>(l) * H, gamma_s, H);
        if (!mk_wait(&a.ready[ph_o(l)], nctas, flags)) return;
        async_copy_wait_all();
        named_sync(1, kMkConsumers);
        act = mk_prologue_rms(st.x, false, gamma_s, H, eps, xq, red);
        mk_run_tiles(sg, seq, a.stages, a.slot_bytes, ring, full, empty, xq, acc_s, flags);
        seq += sg.ntiles;
        if (mk_stop(flags)) return;
        {
            float local = 0.f;
            for (int p = tid; p < (sg.nrows >> 1); p += kMkConsumers) {
                const int b = p / kSwigluBlock, j = p % kSwigluBlock;
                const int gi = 2 * kSwigluBlock * b + j;
                const float gte = mk_value(acc_s, sc_s, gi, act), u = mk_value(acc_s, sc_s, gi + kSwigluBlock, act);
                const float y = __fmul_rn(__fdiv_rn(gte, __fadd_rn(1.0f, exp_cw(-gte))), u);
                __stcg(st.act + (sg.r0 >> 1) + p, y);
                local = fmaxf(local, fabsf(y));
            }
            const float mx = group_max(local, red, kMkWarps, 1);
            if (tid == 0) atomic_max_nonneg(st.absmax + 2 * l + 1, mx);
        }
        mk_signal(&a.ready[ph_gate_up(l)]);

        // ---- down: quantise(act) -> GEMV -> residual ----
        sg = mk_segment(a, 4 * l + SEG_DOWN, cta, nctas);
        mk_fetch_scales(sg, sc_s);
        if (!mk_wait(&a.ready[ph_gate_up(l)], nctas, flags)) return;
        async_copy_wait_all();
        act = mk_prologue_quant(st.act, st.absmax + 2 * l + 1, m.intermediate, xq);
        mk_run_tiles(sg, seq, a.stages, a.slot_bytes, ring, full, empty, xq, acc_s, flags);
        seq += sg.ntiles;
        if (mk_stop(flags)) return;
        for (int i = tid; i < sg.nrows; i += kMkConsumers)
            __stcg(st.x + sg.r0 + i, __fadd_rn(__ldcg(st.x + sg.r0 + i), mk_value(acc_s, sc_s, i, act)));
        mk_signal(&a.ready[ph_down(l)]);
    }

    // ---- LM head: RMSNorm(x) -> quantise -> GEMV -> logits + argmax ----
    const Seg sg = mk_segment(a, 4 * L_layers, cta, nctas);
    mk_fetch_scales(sg, sc_s);
    mk_fetch_gamma(m.norm_final, gamma_s, H);
    if (!mk_wait(&a.ready[ph_down(L_layers - 1)], nctas, flags)) return;
    async_copy_wait_all();
    named_sync(1, kMkConsumers);
    const float act = mk_prologue_rms(st.x, false, gamma_s, H, eps, xq, red);
    mk_run_tiles(sg, seq, a.stages, a.slot_bytes, ring, full, empty, xq, acc_s, flags);
    if (mk_stop(flags)) return;
    unsigned long long best = 0ull;
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
        atomicMax(st.argmax_key, best);
    }
    const int final_phase = 5 * L_layers;
    mk_signal(&a.ready[final_phase]);
    if (cta == 0) {
        if (!mk_wait(&a.ready[final_phase], nctas, flags)) return;
        if (tid == 0) {
            const unsigned long long key = atomicAdd(st.argmax_key, 0ull);
            const int32_t id = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(key & 0xFFFFFFFFull));
            *st.next_token = id;
            *st.token = id;
            *st.position = pos + 1;
        }
    }
}

struct MkPlan {
    MkArgs args;
    int smem;
};

int mk_splits_max(const h4b_model* m) {
    return std::max(1, std::min(64, sm_count() / m->kv_heads));
}

static int plan_persistent(const h4b_model* m, const h4b_state* s, MkPlan* p) {
    int rc = validate(m, s);
    if (rc) return rc;
    if (!s->sync || (reinterpret_cast<uintptr_t>(s->sync) & 15) || !s->attn_partials) return H4B_EINVAL;
    if (m->hidden > kMkMaxHidden) return H4B_EUNSUPPORTED;
    const int q_size = m->heads * m->head_dim;
    const int max_width = std::max(m->hidden, std::max(q_size, m->intermediate));
    if (max_width > kMkMaxWidth) return H4B_EUNSUPPORTED;
    MkArgs& a = p->args;
    a = MkArgs{};
    a.m = *m;
    a.s = *s;
    a.ready = s->sync;
    a.attn_count = s->sync + 5 * m->layers + 2;
    a.attn_chunk = 32;
    a.max_splits = mk_splits_max(m);
    a.xq_bytes = max_width;
    const int nctas = sm_count();
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
    if (!g_prepared) {
        const int prc = prepare_kernels();
        if (prc) return prc;
    }
    MkPlan p;
    int rc = plan_persistent(m, s, &p);
    if (rc) return rc;
    const size_t sync_words = static_cast<size_t>(5 * m->layers + 2) + static_cast<size_t>(m->layers) * m->kv_heads;
    H4B_CUDA_TRY(cudaMemsetAsync(s->sync, 0, sync_words * sizeof(uint32_t), stream));
    H4B_CUDA_TRY(cudaMemsetAsync(s->absmax, 0, 2 * m->layers * sizeof(float), stream));
    H4B_CUDA_TRY(cudaMemsetAsync(s->argmax_key, 0, sizeof(unsigned long long), stream));
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

extern "C" int h4b_decode_persistent(const h4b_model* model, const h4b_state* state, void* stream) {
    return h4b::decode_persistent(model, state, static_cast<cudaStream_t>(stream));
}
