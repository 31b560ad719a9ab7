// Single-token grouped-query attention for decode on sm_100a.
//
// Reference semantics: cpu_kernels/litespark_int4.cpp:160-259 and
// cpu_lightspark.py:389-422 -- s_t = q . k_t / sqrt(d), max-subtracted
// softmax over t <= pos, o = sum_t p_t v_t; q head h reads kv head h / groups.
//
// Split-K ("flash decoding"): grid = (splits, kv_heads, batch). A CTA owns
// one kv head and one chunk of ceil(context / splits) tokens; each of its
// warps owns one q head of the group, so every K/V row it stages serves
// `groups` heads. The chunk is walked in sub-tiles of 64 tokens staged in
// shared memory with one cooperative load each. Per sub-tile a warp scores
// 32 tokens at a time (4 dims per lane, then a transpose-reduce that pairs
// lanes exactly like a butterfly sum), takes a two-pass softmax, and
// accumulates p * v in token order. Sub-tiles fold into the chunk's running
// (m, l, o); chunks are merged either by the last CTA to finish (decode
// path, self-resetting counters) or by a second kernel (the
// reference-compatible entry point). The CPU oracle repeats this order.
//
// In the decode path the kernel also applies, before attending, what
// cpu_lightspark.py:435-440 does between the qkv projection and attention:
// per-head RMSNorm of q and k (divide by sqrt(mean + eps), then scale),
// half-split RoPE at the current position, and the KV-cache append.
#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace h4b {

// Timeline points inside the sub-tile math (phase-trace builds only; the
// persistent kernel sets g_trace_attn around one layer's attention).
#ifdef H4B_PHASE_TRACE
__device__ int g_trace_attn;
#define H4B_TRACE_ATTN(ev) do { if (g_trace_attn) H4B_TRACE(ev); } while (0)
#else
#define H4B_TRACE_ATTN(ev) do { } while (0)
#endif

constexpr int kHeadDim = 128;  // 4 values per lane
// One split result per q head: o[128], m, l, 2 pad floats, so every float4
// store stays 16-byte aligned.
constexpr int kPartialStride = kHeadDim + 4;
constexpr int kSubTile = 64;  // tokens staged per pass
constexpr int kMaxGroups = 8;  // q heads per kv head (one warp each)

// Staged K/V rows are padded by 16 bytes so that lanes reading different
// rows at the same column (one token per lane) hit different bank groups.
template <typename KV>
__host__ __device__ constexpr int kv_row_stride() { return kHeadDim + 16 / static_cast<int>(sizeof(KV)); }
// Shared memory of one staged sub-tile: K and V rows, then one q head per warp.
template <typename KV>
__host__ __device__ constexpr int subtile_smem_bytes() {
    return 2 * kSubTile * kv_row_stride<KV>() * static_cast<int>(sizeof(KV)) + kMaxGroups * kHeadDim * 4;
}

struct AttnArgs {
    const float* q;       // [batch][q_heads][d]  (qkv buffer in the decode path)
    const float* knew;    // [batch][kv_heads][d] raw new key, or null
    const float* vnew;    // [batch][kv_heads][d] new value, or null
    long long q_batch_stride;   // floats between batch entries of q/knew/vnew
    const float* q_norm;  // [d] or null
    const float* k_norm;  // [d] or null
    const float* rope_cos;  // [max_pos][d/2] or null
    const float* rope_sin;
    float eps;
    void* kcache;         // fp32 or fp16 per KV
    void* vcache;
    long long head_stride, time_stride, batch_stride;  // elements
    const int* position;  // per batch entry; context = position + 1
    int context;          // used when position is null
    int capacity;
    int groups, kv_heads, splits;
    float* partials;      // [batch][kv][splits][groups][kPartialStride]
    int* counters;        // [batch][kv] or null (two-kernel merge)
    float* out;           // [batch][q_heads][d]
    long long out_batch_stride;
    float* absmax_out;    // per batch entry or null
};

template <typename KV>
__device__ __forceinline__ float4 load4(const KV* p);
template <>
__device__ __forceinline__ float4 load4<float>(const float* p) {
    return *reinterpret_cast<const float4*>(p);
}
template <>
__device__ __forceinline__ float4 load4<__half>(const __half* p) {
    const uint2 raw = *reinterpret_cast<const uint2*>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
    return make_float4(a.x, a.y, b.x, b.y);
}

template <typename KV>
__device__ __forceinline__ void store4(KV* p, float4 v);
template <>
__device__ __forceinline__ void store4<float>(float* p, float4 v) {
    *reinterpret_cast<float4*>(p) = v;
}
template <>
__device__ __forceinline__ void store4<__half>(__half* p, float4 v) {
    const __half2 a = __floats2half2_rn(v.x, v.y);
    const __half2 b = __floats2half2_rn(v.z, v.w);
    uint2 raw;
    raw.x = *reinterpret_cast<const uint32_t*>(&a);
    raw.y = *reinterpret_cast<const uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = raw;
}

// Eight consecutive K values (16 bytes) as two float4s.
template <typename KV>
__device__ __forceinline__ void load8kv(const KV* p, float4& a, float4& b);
template <>
__device__ __forceinline__ void load8kv<float>(const float* p, float4& a, float4& b) {
    a = *reinterpret_cast<const float4*>(p);
    b = *reinterpret_cast<const float4*>(p + 4);
}
template <>
__device__ __forceinline__ void load8kv<__half>(const __half* p, float4& a, float4& b) {
    const uint4 raw = *reinterpret_cast<const uint4*>(p);
    const float2 x0 = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
    const float2 x1 = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
    const float2 x2 = __half22float2(*reinterpret_cast<const __half2*>(&raw.z));
    const float2 x3 = __half22float2(*reinterpret_cast<const __half2*>(&raw.w));
    a = make_float4(x0.x, x0.y, x1.x, x1.y);
    b = make_float4(x2.x, x2.y, x3.x, x3.y);
}

__device__ __forceinline__ float dot4(float4 a, float4 b) {
    return __fmaf_rn(a.w, b.w, __fmaf_rn(a.z, b.z, __fmaf_rn(a.y, b.y, __fmul_rn(a.x, b.x))));
}

// Constants the per-head norm and RoPE of one lane read: gamma[4 lane ..],
// cos/sin[(4 lane) mod 64 ..]. They are weights and tables, so callers may
// load them before the head itself is ready.
struct HeadConsts {
    float4 g, c, s;
};

__device__ __forceinline__ HeadConsts head_consts(const float* gamma, const float* cs, const float* sn, int lane) {
    HeadConsts k;
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    const int i = (4 * lane) & (kHeadDim / 2 - 1);
    k.g = gamma ? *reinterpret_cast<const float4*>(gamma + 4 * lane) : z;
    k.c = cs ? *reinterpret_cast<const float4*>(cs + i) : z;
    k.s = sn ? *reinterpret_cast<const float4*>(sn + i) : z;
    return k;
}

// Per-head RMSNorm (cpu_lightspark.py:373-379) and half-split RoPE
// (cpu_lightspark.py:381-387) on one 128-wide head held 4 values per lane.
__device__ __forceinline__ float4 norm_rope_with(float4 v, const HeadConsts& k, bool has_gamma, bool has_rope,
                                                 float eps, int lane) {
    if (has_gamma) {
        const float ss = warp_sum(dot4(v, v));
        const float root = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(kHeadDim)), eps));
        v.x = __fmul_rn(__fdiv_rn(v.x, root), k.g.x);
        v.y = __fmul_rn(__fdiv_rn(v.y, root), k.g.y);
        v.z = __fmul_rn(__fdiv_rn(v.z, root), k.g.z);
        v.w = __fmul_rn(__fdiv_rn(v.w, root), k.g.w);
    }
    if (has_rope) {
        float4 other;
        other.x = __shfl_xor_sync(0xffffffffu, v.x, 16);
        other.y = __shfl_xor_sync(0xffffffffu, v.y, 16);
        other.z = __shfl_xor_sync(0xffffffffu, v.z, 16);
        other.w = __shfl_xor_sync(0xffffffffu, v.w, 16);
        const float4 c = k.c, s = k.s;
        if (lane < 16) {  // first half: x1*cos - x2*sin
            v = make_float4(__fsub_rn(__fmul_rn(v.x, c.x), __fmul_rn(other.x, s.x)),
                            __fsub_rn(__fmul_rn(v.y, c.y), __fmul_rn(other.y, s.y)),
                            __fsub_rn(__fmul_rn(v.z, c.z), __fmul_rn(other.z, s.z)),
                            __fsub_rn(__fmul_rn(v.w, c.w), __fmul_rn(other.w, s.w)));
        } else {          // second half: x2*cos + x1*sin
            v = make_float4(__fadd_rn(__fmul_rn(v.x, c.x), __fmul_rn(other.x, s.x)),
                            __fadd_rn(__fmul_rn(v.y, c.y), __fmul_rn(other.y, s.y)),
                            __fadd_rn(__fmul_rn(v.z, c.z), __fmul_rn(other.z, s.z)),
                            __fadd_rn(__fmul_rn(v.w, c.w), __fmul_rn(other.w, s.w)));
        }
    }
    return v;
}

__device__ __forceinline__ float4 norm_rope(float4 v, const float* gamma, const float* cs, const float* sn,
                                            float eps, int lane) {
    return norm_rope_with(v, head_consts(gamma, cs, sn, lane), gamma != nullptr, cs != nullptr, eps, lane);
}

// Combine split results (m_i, l_i, o_i) of one q head into the output, in
// split order. The loads are batched (m and l one split per lane, o eight
// splits at a time) so the merge costs a few L2 round trips, not one per
// split; the arithmetic is the same sequence as a plain loop over splits.
__device__ __forceinline__ float4 merge_splits(const float* base, int splits, int stride, int lane) {
    float mmax = -INFINITY;
    for (int s = lane; s < splits; s += 32) mmax = fmaxf(mmax, __ldcg(base + s * stride + kHeadDim));
    mmax = warp_max(mmax);
    float l = 0.f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    constexpr int kBatch = 8;
    for (int s0 = 0; s0 < splits; s0 += kBatch) {
        float ms[kBatch], ls[kBatch];
        float4 vs[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            const float* p = base + min(s0 + j, splits - 1) * stride;
            ms[j] = __ldcg(p + kHeadDim);
            ls[j] = __ldcg(p + kHeadDim + 1);
            vs[j] = __ldcg(reinterpret_cast<const float4*>(p + 4 * lane));
        }
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            if (s0 + j >= splits || ls[j] == 0.f) continue;
            const float w = exp_cw(ms[j] - mmax);
            l = __fmaf_rn(ls[j], w, l);
            o.x = __fmaf_rn(vs[j].x, w, o.x);
            o.y = __fmaf_rn(vs[j].y, w, o.y);
            o.z = __fmaf_rn(vs[j].z, w, o.z);
            o.w = __fmaf_rn(vs[j].w, w, o.w);
        }
    }
    const float inv = __fdiv_rn(1.0f, l);
    return make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
}

// Sum over lanes of 32 per-lane partials, one per token: afterwards lane l
// holds the total for token l. Each step keeps half of the tokens and adds
// the partner's value for them, so token t is summed over lanes in the same
// pairing order as warp_sum's butterfly (identical bits).
__device__ __forceinline__ float transpose_reduce32(float v[32], int lane) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const bool upper = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < o; ++i) {
            const float keep = upper ? v[i + o] : v[i];
            const float send = upper ? v[i] : v[i + o];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
    }
    return v[0];
}

// Starts the asynchronous copy of sub-tile rows [base, base + n) of one kv
// head's K and V into ks/vs (16-byte pieces spread over `threads` threads),
// leaving out row `skip` (the new token, which arrives from registers).
template <typename KV>
__device__ __forceinline__ void stage_subtile(const KV* kc, const KV* vc, long long time_stride, int base, int n,
                                              int skip, KV* ks, KV* vs, int tid, int threads) {
    constexpr int kRowVecs = kHeadDim * sizeof(KV) / 16;  // a power of two: no runtime division
#pragma unroll 1
    for (int i = tid; i < n * kRowVecs; i += threads) {
        const int r = i / kRowVecs, piece = i % kRowVecs;
        if (base + r == skip) continue;
        const long long src = static_cast<long long>(base + r) * time_stride;
        async_copy16(reinterpret_cast<uint4*>(ks + r * kv_row_stride<KV>()) + piece,
                     reinterpret_cast<const uint4*>(kc + src) + piece);
        async_copy16(reinterpret_cast<uint4*>(vs + r * kv_row_stride<KV>()) + piece,
                     reinterpret_cast<const uint4*>(vc + src) + piece);
    }
}

// Folds one staged sub-tile (n <= kSubTile tokens in ks/vs, rows padded to
// kv_row_stride) into a q head's running (m, l, o).
//
// Scores: the score of a token is the sum of 32 dot4 partials (dims
// 4c..4c+3) added in the pairing order of a warp butterfly sum. Here lane
// (i = lane / 8, t = lane % 8) keeps the 8 q groups c = i + 4j in registers
// and, for token 8 s + t of each step s, forms the partials of its groups,
// adds them through the first three butterfly levels (c^16, c^8, c^4 stay
// inside the lane), and finishes the last two (c^2, c^1) with shuffles
// across lanes 16 and 8 apart -- the same bits as 32 lanes holding one
// group each, with 8x less shared-memory traffic for q. Lane l of round r
// ends with token 32 r + l. Then a two-pass softmax over the sub-tile,
// p * v accumulated in token order (4 dims per lane) and the running merge.
// Tokens past n add p = 0 times a staged row, which leaves every partial
// sum unchanged.
template <typename KV>
__device__ __forceinline__ void attend_subtile(const float* qs, const KV* ks, const KV* vs, int n, float scale,
                                               int lane, float& m, float& l, float4& o) {
    // The loops over rounds, token steps and V tokens stay rolled: this code
    // runs once per layer in the persistent kernel, where every instruction
    // is fetched cold, so a short body executed many times beats a long
    // unrolled one. The arithmetic and its order are the unrolled form's.
    constexpr int S = kv_row_stride<KV>();
    const int qi = lane >> 3, tl = lane & 7;
    const int rounds = n > 32 ? 2 : 1;
    float4 qv[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) qv[j] = *reinterpret_cast<const float4*>(qs + 4 * (qi + 4 * j));
    float p0 = -INFINITY, p1 = -INFINITY;
#pragma unroll 1
    for (int r = 0; r < rounds; ++r) {
        float mine = 0.f;
#pragma unroll 1
        for (int st = 0; st < 4; ++st) {
            const KV* krow = ks + min(32 * r + 8 * st + tl, n - 1) * S + 4 * qi;
            float p[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) p[j] = dot4(qv[j], load4<KV>(krow + 16 * j));
            const float s3 = ((p[0] + p[4]) + (p[2] + p[6])) + ((p[1] + p[5]) + (p[3] + p[7]));
            const float s4 = s3 + __shfl_xor_sync(0xffffffffu, s3, 16);
            const float s5 = s4 + __shfl_xor_sync(0xffffffffu, s4, 8);
            mine = st == qi ? s5 : mine;
        }
        const float sc = (32 * r + lane < n) ? __fmul_rn(mine, scale) : -INFINITY;
        if (r == 0) p0 = sc;
        else p1 = sc;
    }
    H4B_TRACE_ATTN(1510);
    const float mt = warp_max(fmaxf(p0, p1));
    p0 = lane < n ? exp_cw(p0 - mt) : 0.f;
    p1 = 32 + lane < n ? exp_cw(p1 - mt) : 0.f;
    const float lt = warp_sum(p0 + p1);
    H4B_TRACE_ATTN(1511);
    float4 ot = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
    for (int r = 0; r < rounds; ++r) {
        const float pr = r == 0 ? p0 : p1;
        const KV* vrow = vs + 4 * lane;
#pragma unroll 4
        for (int t = 0; t < 32; ++t) {
            const float p = __shfl_sync(0xffffffffu, pr, t);
            const float4 v = load4<KV>(vrow + min(32 * r + t, n - 1) * S);
            ot.x = __fmaf_rn(p, v.x, ot.x);
            ot.y = __fmaf_rn(p, v.y, ot.y);
            ot.z = __fmaf_rn(p, v.z, ot.z);
            ot.w = __fmaf_rn(p, v.w, ot.w);
        }
    }
    H4B_TRACE_ATTN(1512);
    const float mn = fmaxf(m, mt);
    const float c_old = exp_cw(m - mn), c_new = exp_cw(mt - mn);
    l = __fmaf_rn(l, c_old, __fmul_rn(lt, c_new));
    o.x = __fmaf_rn(o.x, c_old, __fmul_rn(ot.x, c_new));
    o.y = __fmaf_rn(o.y, c_old, __fmul_rn(ot.y, c_new));
    o.z = __fmaf_rn(o.z, c_old, __fmul_rn(ot.z, c_new));
    o.w = __fmaf_rn(o.w, c_old, __fmul_rn(ot.w, c_new));
    m = mn;
}

template <typename KV>
__global__ void __launch_bounds__(256) gqa_split_kernel(const AttnArgs a) {
    extern __shared__ __align__(16) uint8_t attn_smem[];
    KV* ks = reinterpret_cast<KV*>(attn_smem);
    KV* vs = ks + kSubTile * kv_row_stride<KV>();
    float* qs = reinterpret_cast<float*>(vs + kSubTile * kv_row_stride<KV>()) + (threadIdx.x >> 5) * kHeadDim;
    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = kvh * a.groups + warp;
    __shared__ int last_flag;
    __shared__ float red[8];

    pdl_wait();
    pdl_trigger();
    const int pos = a.position ? a.position[b] : a.context - 1;
    if (pos < 0 || pos >= a.capacity) {
        if (threadIdx.x == 0 && split == 0 && kvh == 0) report(kStatusBadPosition);
        return;
    }
    const int ctx = pos + 1;
    const int chunk = (ctx + a.splits - 1) / a.splits;
    const int t0 = min(ctx, split * chunk), t1 = min(ctx, t0 + chunk);

    const float* qb = a.q + b * a.q_batch_stride;
    const float* cs = a.rope_cos ? a.rope_cos + static_cast<long long>(pos) * (kHeadDim / 2) : nullptr;
    const float* sn = a.rope_sin ? a.rope_sin + static_cast<long long>(pos) * (kHeadDim / 2) : nullptr;
    float4 q = *reinterpret_cast<const float4*>(qb + static_cast<long long>(h) * kHeadDim + 4 * lane);
    q = norm_rope(q, a.q_norm, cs, sn, a.eps, lane);
    *reinterpret_cast<float4*>(qs + 4 * lane) = q;  // read by every lane in attend_subtile

    KV* kc = static_cast<KV*>(a.kcache) + b * a.batch_stride + kvh * a.head_stride;
    KV* vc = static_cast<KV*>(a.vcache) + b * a.batch_stride + kvh * a.head_stride;
    const bool owns_new = a.knew && t0 <= pos && pos < t1;
    float4 k_new = make_float4(0.f, 0.f, 0.f, 0.f), v_new = k_new;
    if (owns_new) {
        // This CTA's chunk holds the new position: append k (normed, roped) and v.
        if (warp == 0) {
            k_new = *reinterpret_cast<const float4*>(a.knew + b * a.q_batch_stride +
                                                     static_cast<long long>(kvh) * kHeadDim + 4 * lane);
            k_new = norm_rope(k_new, a.k_norm, cs, sn, a.eps, lane);
            store4<KV>(kc + static_cast<long long>(pos) * a.time_stride + 4 * lane, k_new);
        }
        if (warp == a.groups - 1) {
            v_new = *reinterpret_cast<const float4*>(a.vnew + b * a.q_batch_stride +
                                                     static_cast<long long>(kvh) * kHeadDim + 4 * lane);
            store4<KV>(vc + static_cast<long long>(pos) * a.time_stride + 4 * lane, v_new);
        }
    }

    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(kHeadDim)));
    float m = -INFINITY, l = 0.f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int base = t0; base < t1; base += kSubTile) {
        const int n = min(kSubTile, t1 - base);
        __syncthreads();  // the previous sub-tile is consumed
        stage_subtile<KV>(kc, vc, a.time_stride, base, n, owns_new ? pos : -1, ks, vs, threadIdx.x, blockDim.x);
        if (owns_new && pos >= base && pos < base + n) {
            if (warp == 0) store4<KV>(ks + (pos - base) * kv_row_stride<KV>() + 4 * lane, k_new);
            if (warp == a.groups - 1) store4<KV>(vs + (pos - base) * kv_row_stride<KV>() + 4 * lane, v_new);
        }
        async_copy_wait_all();
        __syncthreads();
        attend_subtile<KV>(qs, ks, vs, n, scale, lane, m, l, o);
    }

    float* out_h = a.out + b * a.out_batch_stride + static_cast<long long>(h) * kHeadDim;
    if (a.splits == 1) {
        const float inv = __fdiv_rn(1.0f, l);
        const float4 r = make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
        *reinterpret_cast<float4*>(out_h + 4 * lane) = r;
        if (a.absmax_out) {
            const float mx = warp_max(fmaxf(fmaxf(fabsf(r.x), fabsf(r.y)), fmaxf(fabsf(r.z), fabsf(r.w))));
            if (lane == 0) atomic_max_nonneg(a.absmax_out + b, mx);
        }
        return;
    }

    const int stride = kPartialStride;
    float* part = a.partials + ((static_cast<long long>(b) * a.kv_heads + kvh) * a.splits + split) * a.groups * stride;
    float* mine = part + warp * stride;
    *reinterpret_cast<float4*>(mine + 4 * lane) = o;
    if (lane == 0) {
        mine[kHeadDim] = m;
        mine[kHeadDim + 1] = l;
    }
    if (!a.counters) return;

    // Last CTA of this (batch, kv head) merges all splits.
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        int* counter = a.counters + b * a.kv_heads + kvh;
        const int prev = atomicAdd(counter, 1);
        last_flag = (prev == a.splits - 1);
        if (last_flag) *counter = 0;
    }
    __syncthreads();
    if (!last_flag) return;
    __threadfence();
    const float* base = a.partials + (static_cast<long long>(b) * a.kv_heads + kvh) * a.splits * a.groups * stride +
                        warp * stride;
    const float4 r = merge_splits(base, a.splits, a.groups * stride, lane);
    *reinterpret_cast<float4*>(out_h + 4 * lane) = r;
    if (a.absmax_out) {
        const float mx = warp_max(fmaxf(fmaxf(fabsf(r.x), fabsf(r.y)), fmaxf(fabsf(r.z), fabsf(r.w))));
        if (lane == 0) red[warp] = mx;
        __syncthreads();
        if (threadIdx.x == 0) {
            float t = red[0];
            for (int w = 1; w < a.groups; ++w) t = fmaxf(t, red[w]);
            atomic_max_nonneg(a.absmax_out + b, t);
        }
    }

}

__global__ void __launch_bounds__(256) gqa_merge_kernel(const AttnArgs a) {
    const int kvh = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = kvh * a.groups + warp;
    const int stride = kPartialStride;
    pdl_wait();
    pdl_trigger();
    const float* base = a.partials + (static_cast<long long>(b) * a.kv_heads + kvh) * a.splits * a.groups * stride +
                        warp * stride;
    const float4 r = merge_splits(base, a.splits, a.groups * stride, lane);
    *reinterpret_cast<float4*>(a.out + b * a.out_batch_stride + static_cast<long long>(h) * kHeadDim + 4 * lane) = r;
}

int launch_attention(const AttnArgs& a, int kv_dtype, int batch, cudaStream_t stream, bool pdl) {
    if (a.groups < 1 || a.groups > kMaxGroups || a.splits < 1 || a.kv_heads < 1 || batch < 1) return H4B_EINVAL;
    {  // the shared-memory opt-in of gqa_split_kernel<float> on this device
        const int rc = prepare_kernels();
        if (rc) return rc;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.splits, a.kv_heads, batch);
    cfg.blockDim = dim3(32 * a.groups);
    cfg.dynamicSmemBytes = kv_dtype == 0 ? subtile_smem_bytes<float>() : subtile_smem_bytes<__half>();
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    if (kv_dtype == 0) H4B_CUDA_TRY(cudaLaunchKernelEx(&cfg, gqa_split_kernel<float>, a));
    else H4B_CUDA_TRY(cudaLaunchKernelEx(&cfg, gqa_split_kernel<__half>, a));
    if (a.splits > 1 && !a.counters) {
        cfg.gridDim = dim3(1, a.kv_heads, batch);
        cfg.dynamicSmemBytes = 0;
        H4B_CUDA_TRY(cudaLaunchKernelEx(&cfg, gqa_merge_kernel, a));
    }
    return 0;
}

}  // namespace h4b

extern "C" int h4b_gqa_decode(const float* query, const float* keys, const float* values, float* scores,
                              float* output, int context, int kv_heads, int groups, int head_dim,
                              int score_stride, void* stream) {
    if (!query || !keys || !values || !scores || !output) return H4B_EINVAL;
    if (head_dim != h4b::kHeadDim) return H4B_EUNSUPPORTED;
    if (context < 1 || context > score_stride || kv_heads < 1 || groups < 1 || groups > 8) return H4B_EINVAL;
    h4b::AttnArgs a = {};
    a.q = query;
    a.kcache = const_cast<float*>(keys);
    a.vcache = const_cast<float*>(values);
    a.head_stride = head_dim;
    a.time_stride = static_cast<long long>(kv_heads) * head_dim;
    a.context = context;
    a.capacity = context;
    a.groups = groups;
    a.kv_heads = kv_heads;
    // The reference hands over q_heads * score_stride floats of scratch; keep
    // the split partials (kPartialStride floats per head and split) inside it.
    const int fit = score_stride / h4b::kPartialStride;
    a.splits = std::max(1, std::min({fit, 64, (context + 63) / 64}));
    a.partials = scores;
    a.out = output;
    return h4b::launch_attention(a, 0, 1, static_cast<cudaStream_t>(stream), false);
}

// ---------------------------------------------------------------------------
// Allocation-free variant of h4b_gqa_decode.
//
// The split partials live in this file-scope array instead of caller
// scratch. Every GPU that loads the library holds it (1 MiB) until the
// process exits. Host code must not hand the array's name to a kernel: on
// the host it is only a stand-in, so its device address is looked up once
// per device with cudaGetSymbolAddress (with that device current) and cached.
namespace h4b {

constexpr int kNoAllocScratchFloats = 256 * 1024;  // 1 MiB
static __device__ __align__(256) float g_noalloc_partials[kNoAllocScratchFloats];

static std::atomic<float*> g_noalloc_ptr[kMaxDevices];

// The device address of the static array on the current device. Looked up
// with cudaGetSymbolAddress on the first call per device and cached; a failed
// lookup (e.g. a first call made inside a stream capture) is not cached, so
// the next call tries again.
static int noalloc_scratch(float** out) {
    int dev = 0;
    H4B_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return H4B_EUNSUPPORTED;
    float* ptr = g_noalloc_ptr[dev].load(std::memory_order_acquire);
    if (!ptr) {
        void* addr = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&addr, g_noalloc_partials);
        if (e != cudaSuccess) return static_cast<int>(e);
        if (!addr) return H4B_EUNSUPPORTED;
        ptr = static_cast<float*>(addr);
        g_noalloc_ptr[dev].store(ptr, std::memory_order_release);
    }
    *out = ptr;
    return 0;
}

}  // namespace h4b

extern "C" int h4b_gqa_decode_noalloc(const float* query, const float* keys, const float* values, float* output,
                                      int context, int kv_heads, int groups, int head_dim, void* stream) {
    if (!query || !keys || !values || !output) return H4B_EINVAL;
    if (head_dim != h4b::kHeadDim) return H4B_EUNSUPPORTED;
    if (context < 1 || kv_heads < 1 || groups < 1 || groups > 8) return H4B_EINVAL;
    const long long per_split = static_cast<long long>(kv_heads) * groups * h4b::kPartialStride;
    if (per_split > h4b::kNoAllocScratchFloats) return H4B_ETOOBIG;
    float* scratch = nullptr;
    const int rc = h4b::noalloc_scratch(&scratch);
    if (rc) return rc;
    h4b::AttnArgs a = {};
    a.q = query;
    a.kcache = const_cast<float*>(keys);
    a.vcache = const_cast<float*>(values);
    a.head_stride = head_dim;
    a.time_stride = static_cast<long long>(kv_heads) * head_dim;
    a.context = context;
    a.capacity = context;
    a.groups = groups;
    a.kv_heads = kv_heads;
    // Same split rule as h4b_gqa_decode, with the static array as the room.
    const int fit = static_cast<int>(h4b::kNoAllocScratchFloats / per_split);
    a.splits = std::max(1, std::min({fit, 64, (context + 63) / 64}));
    a.partials = scratch;  // every slot read is written earlier in the same call
    a.out = output;
    return h4b::launch_attention(a, 0, 1, static_cast<cudaStream_t>(stream), false);
}
