// Single-token grouped-query attention for decode on sm_100a.
//
// Reference semantics: cpu_kernels/litespark_int4.cpp:160-259 and
// cpu_lightspark.py:389-422 -- s_t = q . k_t / sqrt(d), max-subtracted
// softmax over t <= pos, o = sum_t p_t v_t; q head h reads kv head h / groups.
//
// Split-K ("flash decoding"): grid = (splits, kv_heads, batch). A CTA owns
// one kv head and one slice of the context; each of its warps owns one q
// head of the group, so every K/V row it streams serves `groups` heads.
// Each warp keeps an online softmax (m, l, o) and the slices are merged
// either by the last CTA to finish (decode path, self-resetting counters)
// or by a second kernel (the reference-compatible entry point).
//
// In the decode path the kernel also applies, before attending, what
// cpu_lightspark.py:435-440 does between the qkv projection and attention:
// per-head RMSNorm of q and k (divide by sqrt(mean + eps), then scale),
// half-split RoPE at the current position, and the KV-cache append.
#include <algorithm>

#include "common.cuh"

namespace h4b {

constexpr int kHeadDim = 128;  // 4 values per lane
// One split result per q head: o[128], m, l, 2 pad floats, so every float4
// store stays 16-byte aligned.
constexpr int kPartialStride = kHeadDim + 4;

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

__device__ __forceinline__ float dot4(float4 a, float4 b) {
    return __fmaf_rn(a.w, b.w, __fmaf_rn(a.z, b.z, __fmaf_rn(a.y, b.y, __fmul_rn(a.x, b.x))));
}

// Per-head RMSNorm (cpu_lightspark.py:373-379) and half-split RoPE
// (cpu_lightspark.py:381-387) on one 128-wide head held 4 values per lane.
__device__ __forceinline__ float4 norm_rope(float4 v, const float* gamma, const float* cs, const float* sn,
                                            float eps, int lane) {
    if (gamma) {
        const float ss = warp_sum(dot4(v, v));
        const float root = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(kHeadDim)), eps));
        const float4 g = *reinterpret_cast<const float4*>(gamma + 4 * lane);
        v.x = __fmul_rn(__fdiv_rn(v.x, root), g.x);
        v.y = __fmul_rn(__fdiv_rn(v.y, root), g.y);
        v.z = __fmul_rn(__fdiv_rn(v.z, root), g.z);
        v.w = __fmul_rn(__fdiv_rn(v.w, root), g.w);
    }
    if (cs) {
        float4 other;
        other.x = __shfl_xor_sync(0xffffffffu, v.x, 16);
        other.y = __shfl_xor_sync(0xffffffffu, v.y, 16);
        other.z = __shfl_xor_sync(0xffffffffu, v.z, 16);
        other.w = __shfl_xor_sync(0xffffffffu, v.w, 16);
        const int i = (4 * lane) & (kHeadDim / 2 - 1);
        const float4 c = *reinterpret_cast<const float4*>(cs + i);
        const float4 s = *reinterpret_cast<const float4*>(sn + i);
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

// Combine split results (m_i, l_i, o_i) of one q head into the output.
__device__ __forceinline__ float4 merge_splits(const float* base, int splits, int stride, int lane) {
    float mmax = -INFINITY;
    for (int s = 0; s < splits; ++s) mmax = fmaxf(mmax, __ldcg(base + s * stride + kHeadDim));
    float l = 0.f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < splits; ++s) {
        const float* p = base + s * stride;
        const float ls = __ldcg(p + kHeadDim + 1);
        if (ls == 0.f) continue;
        const float w = exp_cw(__ldcg(p + kHeadDim) - mmax);
        l = __fmaf_rn(ls, w, l);
        const float4 v = __ldcg(reinterpret_cast<const float4*>(p + 4 * lane));
        o.x = __fmaf_rn(v.x, w, o.x);
        o.y = __fmaf_rn(v.y, w, o.y);
        o.z = __fmaf_rn(v.z, w, o.z);
        o.w = __fmaf_rn(v.w, w, o.w);
    }
    const float inv = __fdiv_rn(1.0f, l);
    return make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
}

template <typename KV>
__global__ void __launch_bounds__(256) gqa_split_kernel(const AttnArgs a) {
    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = kvh * a.groups + warp;
    const int q_heads = a.kv_heads * a.groups;
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

    KV* kc = static_cast<KV*>(a.kcache) + b * a.batch_stride + kvh * a.head_stride;
    KV* vc = static_cast<KV*>(a.vcache) + b * a.batch_stride + kvh * a.head_stride;
    if (a.knew && t0 <= pos && pos < t1) {
        // This CTA's slice holds the new position: append k (normed, roped) and v.
        if (warp == 0) {
            float4 k = *reinterpret_cast<const float4*>(a.knew + b * a.q_batch_stride +
                                                         static_cast<long long>(kvh) * kHeadDim + 4 * lane);
            k = norm_rope(k, a.k_norm, cs, sn, a.eps, lane);
            store4<KV>(kc + static_cast<long long>(pos) * a.time_stride + 4 * lane, k);
        }
        if (warp == a.groups - 1) {
            const float4 v = *reinterpret_cast<const float4*>(a.vnew + b * a.q_batch_stride +
                                                               static_cast<long long>(kvh) * kHeadDim + 4 * lane);
            store4<KV>(vc + static_cast<long long>(pos) * a.time_stride + 4 * lane, v);
        }
        __syncthreads();
    }

    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(kHeadDim)));
    float m = -INFINITY, l = 0.f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    constexpr int U = 4;
    for (int t = t0; t < t1; t += U) {
        float4 kk[U], vv[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int tt = min(t + u, t1 - 1);
            kk[u] = load4<KV>(kc + static_cast<long long>(tt) * a.time_stride + 4 * lane);
            vv[u] = load4<KV>(vc + static_cast<long long>(tt) * a.time_stride + 4 * lane);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (t + u >= t1) break;
            const float s = __fmul_rn(warp_sum(dot4(q, kk[u])), scale);
            const float mn = fmaxf(m, s);
            const float corr = exp_cw(m - mn);
            const float p = exp_cw(s - mn);
            l = __fmaf_rn(l, corr, p);
            o.x = __fmaf_rn(o.x, corr, __fmul_rn(p, vv[u].x));
            o.y = __fmaf_rn(o.y, corr, __fmul_rn(p, vv[u].y));
            o.z = __fmaf_rn(o.z, corr, __fmul_rn(p, vv[u].z));
            o.w = __fmaf_rn(o.w, corr, __fmul_rn(p, vv[u].w));
            m = mn;
        }
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
    (void)q_heads;
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
    if (a.groups < 1 || a.groups > 8 || a.splits < 1 || a.kv_heads < 1 || batch < 1) return H4B_EINVAL;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.splits, a.kv_heads, batch);
    cfg.blockDim = dim3(32 * a.groups);
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
