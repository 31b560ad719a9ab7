// Batched decode attention on the 5th-generation tensor cores (tcgen05
// kind::f16, fp32 accumulators in tensor memory, K/V tiles fed by TMA).
//
// Scope: an fp16 K/V cache, head_dim 128, 4 q heads per kv head; batched
// decode asks for it with h4b_batch_state.attn_kernel (the exact fp32
// kernel of attention.cu stays the default there).
//
// One query per sequence means only the group's 4 q heads share a K/V tile,
// too few rows for an MMA. So the keys are the MMA's M and the heads its N:
//   S^T [128 keys x 16] = K_tile [128 keys x 128 d] . q^T [128 d x 16]
//   O^T [128 d x 16]   += V_tile^T [128 d x 128 keys] . P^T [128 keys x 16]
// K is read K-major as the A operand; V, laid out [key][d] in the cache, is
// the A operand read MN-major; q^T and P^T are K-major B operands in shared
// memory.
//
// Precision (the tolerance contract, as the prefill's tensor-core path): the
// fp16 K and V are the cache's own values; q and p enter as (hi, lo) fp16
// pairs. The (hi, lo) halves share one MMA: B rows 0-3 carry the 4 heads' hi
// parts, rows 4-7 their lo parts (8-15 zero), so S^T columns h and 4 + h and
// O^T columns h and 4 + h hold the two fp32 partial products of head h, added
// by the key warps. Softmax in base 2 with a lazily moved reference maximum
// (p <= 2^15).
//
// Work split: one CTA per (split, kv head, sequence); a split takes whole
// 128-key tiles of its sequence's context. Warps 0-3 are the key warps:
// thread = TMEM lane = key row of S^T (and d row of O^T), 4 loads K tiles and
// owns the tensor memory, 5 loads V tiles, 6 issues the MMAs. Per tile j
// (S^T and P^T double-buffered, b = j % 2):
//   MMA:  S^T[b] = K_j [qhi qlo]^T (8 MMAs)              -> s_full[b], k_empty
//   keys: load S^T row; per-head maxima over the tile (warp maxima exchanged
//         through shared memory, mx_full[b]); p; P^T[b] (hi, lo) -> p_full[b]
//   MMA:  O^T += V_j^T [Phi Plo]^T (8 MMAs)              -> o_full, v_empty
// The MMA thread issues P.V for tile j then S for tile j + 2 (S^T[b] was read
// before p_full[b]; s_full for tile j implies P.V j - 2 completed).
// The split's result is written as a partial (unnormalised o, m, l) in the
// split kernel's layout and merged by gqa_merge_kernel, or, with one split,
// normalised into the output directly.
//
// Every wait is bounded (mbar_wait); a role that gives up marks the CTA
// failed and stops, the producers wait for their copies, and the tensor
// memory is freed after the MMA thread's last commit has arrived.

namespace h4b {

constexpr int kDtcKeys = 128;                        // keys per tile (M of S^T, K of the P.V MMAs)
constexpr int kDtcN = 16;                            // MMA N: q heads, padded
constexpr int kDtcGroups = 4;                        // q heads per kv head
constexpr int kDtcDim = 128;
constexpr int kDtcStages = 2;
constexpr int kDtcKeyWarps = 4, kDtcKWarp = 4, kDtcVWarp = 5, kDtcMmaWarp = 6;
constexpr int kDtcThreads = 32 * 7;

// Shared memory (1024-byte aligned regions):
//   K, V: [stage][d half][128 keys x 128 B]     kDtcStages x 32 KB each
//   q^T:  [d half][16 rows x 128 B]              2 x 2 KB (rows: 4 hi, 4 lo, 8 zero)
//   P^T:  [buffer][key half][16 x 128 B]        4 x 2 KB (the same rows)
constexpr int kDtcHalfTile = kDtcKeys * 128;         // 16 KB
constexpr int kDtcSmallTile = kDtcN * 128;           // 2 KB
constexpr int kDtcKOff = 0;
constexpr int kDtcVOff = kDtcKOff + kDtcStages * 2 * kDtcHalfTile;
constexpr int kDtcQOff = kDtcVOff + kDtcStages * 2 * kDtcHalfTile;
constexpr int kDtcPOff = kDtcQOff + 2 * kDtcSmallTile;
constexpr int kDtcMxOff = kDtcPOff + 4 * kDtcSmallTile;  // [2][4 warps][16] floats, then [4][16] row sums
constexpr int kDtcBarOff = kDtcMxOff + 2 * kDtcKeyWarps * kDtcN * 4 + kDtcKeyWarps * kDtcN * 4;
constexpr int kDtcBarBytes = 256;
constexpr int kDtcSmem = kDtcBarOff + kDtcBarBytes + 1024;
static_assert(kDtcSmem <= 232448, "shared memory per CTA");
static_assert((4 * kDtcStages + 11) * 8 + 8 <= kDtcBarBytes, "barrier area");

// Tensor memory: S^T[0], S^T[1], O^T (16 columns each).
constexpr uint32_t kDtcTmemCols = 64;
constexpr uint32_t kDtcSCol = 0, kDtcOCol = 2 * kDtcN;

// kind::f16, D f32: S^T = A K-major (K tile) x B K-major (q^T); O^T = A
// MN-major (V tile, bit 15) x B K-major (P^T). N = 16, M = 128.
constexpr uint32_t kDtcIdescS = (1u << 4) | (static_cast<uint32_t>(kDtcN >> 3) << 17) |
                                (static_cast<uint32_t>(kDtcKeys >> 4) << 24);
constexpr uint32_t kDtcIdescPV = (1u << 4) | (1u << 15) | (static_cast<uint32_t>(kDtcN >> 3) << 17) |
                                 (static_cast<uint32_t>(kDtcDim >> 4) << 24);

// Byte offset of fp16 element (row r, column c) inside a K-major 128-byte-
// swizzled region of 128-byte rows (64 fp16 per row).
__device__ __forceinline__ int sw128_elem(int r, int c) {
    return (r >> 3) * 1024 + (r & 7) * 128 + ((((c >> 3) ^ (r & 7))) << 4) + (c & 7) * 2;
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int x, int y, int z, int w,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
        "[%6];"
        ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_addr(bar))
        : "memory");
}

struct DtcArgs {
    const float* q;          // normalised, rotated q rows [batch][q_heads * d] (stride q_stride)
    long long q_stride;
    const int32_t* position; // per sequence: context = position + 1
    int splits, kv_heads, capacity;
    float* partials;         // [batch][kv][splits][groups][kPartialStride]
    float* out;              // [batch][q_heads][d] (stride out_stride)
    long long out_stride;
};

__global__ void __launch_bounds__(kDtcThreads, 1)
    decode_attention_tc_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                               const DtcArgs a) {
    extern __shared__ uint8_t dtc_smem_raw[];
    uint8_t* smem = dtc_smem_raw + ((1024u - (smem_addr(dtc_smem_raw) & 1023u)) & 1023u);
    uint64_t* k_full = reinterpret_cast<uint64_t*>(smem + kDtcBarOff);
    uint64_t* k_empty = k_full + kDtcStages;
    uint64_t* v_full = k_empty + kDtcStages;
    uint64_t* v_empty = v_full + kDtcStages;
    uint64_t* s_full = v_empty + kDtcStages;  // [2]
    uint64_t* p_full = s_full + 2;             // [2]
    uint64_t* mx_full = p_full + 2;            // [2] the key warps' tile maxima written
    uint64_t* o_full = mx_full + 2;
    uint64_t* q_ready = o_full + 1;
    uint64_t* mma_done = q_ready + 1;
    uint64_t* sum_full = mma_done + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sum_full + 1);
    volatile int* failed = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* mx = reinterpret_cast<float*>(smem + kDtcMxOff);                       // [2][4][16]
    float* lsum = mx + 2 * kDtcKeyWarps * kDtcN;                                  // [4][16]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int pos = a.position[b];
    const int ctx = pos >= 0 && pos < a.capacity ? pos + 1 : 0;
    // this split's keys [t0, t1): whole tiles of the context
    const int ctx_tiles = (ctx + kDtcKeys - 1) / kDtcKeys;
    const int tile0 = static_cast<int>(static_cast<long long>(split) * ctx_tiles / a.splits);
    const int tile1 = static_cast<int>(static_cast<long long>(split + 1) * ctx_tiles / a.splits);
    const int tiles = tile1 - tile0;
    const int t1 = min(ctx, tile1 * kDtcKeys);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kDtcStages; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], kDtcKeyWarps);
            mbar_init(&mx_full[i], kDtcKeyWarps);
        }
        mbar_init(o_full, 1);
        mbar_init(q_ready, kDtcKeyWarps);
        mbar_init(mma_done, 1);
        mbar_init(sum_full, kDtcKeyWarps);
        *failed = wait_failed_before() ? 1 : 0;
        fence_mbar_init();
    }
    if (warp == kDtcKWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_addr(tmem_slot)), "r"(kDtcTmemCols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    auto k_half = [&](int s, int half) { return smem + kDtcKOff + (s * 2 + half) * kDtcHalfTile; };
    auto v_half = [&](int s, int half) { return smem + kDtcVOff + (s * 2 + half) * kDtcHalfTile; };
    auto q_tile = [&](int half) { return smem + kDtcQOff + half * kDtcSmallTile; };
    auto p_tile = [&](int buf, int half) { return smem + kDtcPOff + (buf * 2 + half) * kDtcSmallTile; };

    if (warp == kDtcKWarp || warp == kDtcVWarp) {
        if (lane == 0) {  // TMA producer of the K (or V) tiles of this split
            const bool is_k = warp == kDtcKWarp;
            const CUtensorMap* map = is_k ? &kmap : &vmap;
            uint64_t* full = is_k ? k_full : v_full;
            uint64_t* empty = is_k ? k_empty : v_empty;
            int issued = 0;
            if (!*failed) {
                asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
                for (int j = 0; j < tiles; ++j) {
                    const int s = j % kDtcStages;
                    if (*failed) break;
                    if (j >= kDtcStages && !mbar_wait(&empty[s], (j / kDtcStages - 1) & 1)) {
                        *failed = 1;
                        break;
                    }
                    uint8_t* dst0 = is_k ? k_half(s, 0) : v_half(s, 0);
                    uint8_t* dst1 = is_k ? k_half(s, 1) : v_half(s, 1);
                    mbar_arrive_expect_tx(&full[s], 2 * kDtcHalfTile);
                    tma_load_4d(dst0, map, 0, (tile0 + j) * kDtcKeys, kvh, b, &full[s]);
                    tma_load_4d(dst1, map, kDtcDim / 2, (tile0 + j) * kDtcKeys, kvh, b, &full[s]);
                    issued = j + 1;
                }
            }
            for (int j = issued > kDtcStages ? issued - kDtcStages : 0; j < issued; ++j)
                mbar_wait(&full[j % kDtcStages], (j / kDtcStages) & 1);
        }
    } else if (warp == kDtcMmaWarp) {
        if (lane == 0) {
            auto issue_s = [&](int j) -> bool {
                const int s = j % kDtcStages, bb = j & 1;
                if (*failed) return false;
                if (!mbar_wait(&k_full[s], (j / kDtcStages) & 1)) return false;
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < kDtcDim / 16; ++kk) {  // 16 dims = 32 bytes = +2 in the address field
                    const uint64_t ad = sw128_desc(k_half(s, kk >> 2)) + 2 * (kk & 3);
                    const uint64_t bd = sw128_desc(q_tile(kk >> 2)) + 2 * (kk & 3);
                    tc_mma_f16(tmem + kDtcSCol + bb * kDtcN, ad, bd, kDtcIdescS, kk != 0);
                }
                tc_commit(&k_empty[s]);
                tc_commit(&s_full[bb]);
                return true;
            };
            auto issue_pv = [&](int j) -> bool {
                const int s = j % kDtcStages, bb = j & 1;
                if (*failed) return false;
                if (!mbar_wait(&p_full[bb], (j >> 1) & 1)) return false;
                if (!mbar_wait(&v_full[s], (j / kDtcStages) & 1)) return false;
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < kDtcKeys / 16; ++kk) {
                    // A: V^T, 16 keys = 2 groups of 8 key rows = 2048 bytes on, the other
                    // 64 dims one half tile on; B: P^T, 16 keys = 32 bytes along its rows
                    const uint64_t ad = sw128_mn_desc(v_half(s, 0) + (kk & 7) * 2048, kDtcHalfTile);
                    const uint64_t bd = sw128_desc(p_tile(bb, kk >> 2)) + 2 * (kk & 3);
                    tc_mma_f16(tmem + kDtcOCol, ad, bd, kDtcIdescPV, (j | kk) != 0);
                }
                tc_commit(&v_empty[s]);
                tc_commit(o_full);
                return true;
            };
            bool ok = true;
            if (tiles > 0) {
                ok = !*failed && mbar_wait(q_ready, 0);
                ok = ok && issue_s(0) && (tiles < 2 || issue_s(1));
                for (int j = 0; ok && j < tiles; ++j) ok = issue_pv(j) && (j + 2 >= tiles || issue_s(j + 2));
            }
            if (!ok) *failed = 1;
            tc_commit(mma_done);
        }
    } else {  // key warps: thread = TMEM lane 32 warp + lane (key row of S^T, d row of O^T)
        const int row = 32 * warp + lane;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(32 * warp) << 16);
        // q^T: rows h = hi, 4 + h = lo of the group's heads, rows 8..15 zero;
        // P^T's zero rows 8..15
        {
            const float* qh = a.q + static_cast<long long>(b) * a.q_stride + static_cast<long long>(kvh) * kDtcGroups * kDtcDim;
            for (int e = threadIdx.x; e < kDtcGroups * kDtcDim / 2; e += 32 * kDtcKeyWarps) {
                const int h = e / (kDtcDim / 2), d = 2 * (e % (kDtcDim / 2));
                float2 x = make_float2(0.f, 0.f);
                if (ctx > 0) x = *reinterpret_cast<const float2*>(qh + h * kDtcDim + d);
                uint32_t hi, lo;
                split_pair(x.x, x.y, hi, lo);
                *reinterpret_cast<uint32_t*>(q_tile(d >> 6) + sw128_elem(h, d & 63)) = hi;
                *reinterpret_cast<uint32_t*>(q_tile(d >> 6) + sw128_elem(kDtcGroups + h, d & 63)) = lo;
            }
            constexpr int kZeroRows = kDtcN - 2 * kDtcGroups;
            for (int e = threadIdx.x; e < 6 * kZeroRows * 32; e += 32 * kDtcKeyWarps) {
                // 6 tiles (q^T halves, P^T buffers x halves), rows 8..15, 32 column pairs each
                const int c = 2 * (e % 32), r = 2 * kDtcGroups + (e / 32) % kZeroRows, t = e / (32 * kZeroRows);
                uint8_t* tile = t < 2 ? q_tile(t) : p_tile((t - 2) >> 1, (t - 2) & 1);
                *reinterpret_cast<uint32_t*>(tile + sw128_elem(r, c)) = 0u;
            }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(q_ready);

        const float score_scale = 1.4426950408889634f * 0.08838834764831845f;  // log2(e) / sqrt(128)
        float m_ref[kDtcGroups], lt[kDtcGroups];
#pragma unroll
        for (int h = 0; h < kDtcGroups; ++h) {
            m_ref[h] = -INFINITY;
            lt[h] = 0.f;
        }
        bool ok = true;
        for (int j = 0; j < tiles && ok; ++j) {
            const int bb = j & 1, kbase = (tile0 + j) * kDtcKeys;
            ok = __all_sync(0xffffffffu, !*failed && mbar_wait(&s_full[bb], (j >> 1) & 1));
            if (!ok) break;
            tc_fence_after();
            float sv[kDtcN];
            tmem_ld16_nowait(lane_base + kDtcSCol + bb * kDtcN, sv, 0);
            tmem_wait_regs(sv);
#pragma unroll
            for (int h = 0; h < kDtcGroups; ++h) sv[h] = __fadd_rn(sv[h], sv[kDtcGroups + h]);  // q hi + q lo parts
            const bool in = kbase + row < t1;
            // the tile's per-head maxima: warp maxima, exchanged
            float wm[kDtcGroups];
#pragma unroll
            for (int h = 0; h < kDtcGroups; ++h) {
                sv[h] = in ? sv[h] : -INFINITY;
                wm[h] = warp_max(sv[h]);
            }
            float* slot = mx + bb * kDtcKeyWarps * kDtcN;
            if (lane < kDtcGroups)
                slot[warp * kDtcN + lane] = lane == 0 ? wm[0] : (lane == 1 ? wm[1] : (lane == 2 ? wm[2] : wm[3]));
            __syncwarp();
            if (lane == 0) mbar_arrive(&mx_full[bb]);
            ok = __all_sync(0xffffffffu, !*failed && mbar_wait(&mx_full[bb], (j >> 1) & 1));
            if (!ok) break;
            float tmax[kDtcGroups];
            bool need = false;
#pragma unroll
            for (int h = 0; h < kDtcGroups; ++h) {
                float t = fmaxf(fmaxf(slot[h], slot[kDtcN + h]), fmaxf(slot[2 * kDtcN + h], slot[3 * kDtcN + h]));
                tmax[h] = t * score_scale;
                need = need || (tmax[h] > m_ref[h] + kPtcSlack && m_ref[h] != -INFINITY);
            }
            if (need) {  // uniform: every key warp read the same maxima
                ok = __all_sync(0xffffffffu, !*failed && mbar_wait(o_full, (j - 1) & 1));
                if (!ok) break;
                tc_fence_after();
                float alpha[kDtcGroups];
#pragma unroll
                for (int h = 0; h < kDtcGroups; ++h)
                    alpha[h] = tmax[h] > m_ref[h] + kPtcSlack && m_ref[h] != -INFINITY ? ex2_approx(m_ref[h] - tmax[h])
                                                                                     : 1.f;
                float o[kDtcN];
                tmem_ld16_nowait(lane_base + kDtcOCol, o, 0);
                tmem_wait_regs(o);
#pragma unroll
                for (int h = 0; h < kDtcGroups; ++h) {
                    o[h] *= alpha[h];
                    o[kDtcGroups + h] *= alpha[h];
                }
                tmem_st16(lane_base + kDtcOCol, o, 0);
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
#pragma unroll
                for (int h = 0; h < kDtcGroups; ++h) lt[h] *= alpha[h];
            }
            // p = 2^(s * scale - (m_ref - 8)) in P^T (hi, lo)
#pragma unroll
            for (int h = 0; h < kDtcGroups; ++h) {
                if (tmax[h] > m_ref[h] + kPtcSlack) m_ref[h] = tmax[h];
                const float nbase = m_ref[h] == -INFINITY ? 0.f : kPtcOffset - m_ref[h];
                const float p = ex2_approx(__fmaf_rn(sv[h], score_scale, nbase));
                lt[h] += p;
                const __half hi = __float2half_rn(p);
                const __half lo = __float2half_rn(p - __half2float(hi));
                *reinterpret_cast<__half*>(p_tile(bb, row >> 6) + sw128_elem(h, row & 63)) = hi;
                *reinterpret_cast<__half*>(p_tile(bb, row >> 6) + sw128_elem(kDtcGroups + h, row & 63)) = lo;
            }
            if (j == tiles - 1 && t1 < kbase + kDtcKeys) {
                // keys past the context: p = 0, and their V rows zeroed (a
                // cache entry never written could hold NaN); s_full for this
                // tile implies P.V j - 2 completed, so v_full's phase is this tile's
                const int s = j % kDtcStages;
                ok = __all_sync(0xffffffffu, !*failed && mbar_wait(&v_full[s], (j / kDtcStages) & 1));
                if (!ok) break;
                const int first = t1 - kbase;
                const int chunks = (kDtcKeys - first) * 8;
                for (int t = threadIdx.x; t < 2 * chunks; t += 32 * kDtcKeyWarps) {
                    const int half = t / chunks, idx = t % chunks;
                    *reinterpret_cast<uint4*>(v_half(s, half) + (first + idx / 8) * 128 + (idx % 8) * 16) =
                        make_uint4(0u, 0u, 0u, 0u);
                }
            }
            fence_proxy_async_smem();  // P^T (and zeroed V rows) -> the tensor cores
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[bb]);
        }
        // the heads' row sums over the split's keys: warp sums, then the four warps
        float ls[kDtcGroups];
#pragma unroll
        for (int h = 0; h < kDtcGroups; ++h) ls[h] = warp_sum(lt[h]);
        if (lane < kDtcGroups)
            lsum[warp * kDtcN + lane] = lane == 0 ? ls[0] : (lane == 1 ? ls[1] : (lane == 2 ? ls[2] : ls[3]));
        __syncwarp();
        if (lane == 0) mbar_arrive(sum_full);
        const bool have_sum = __all_sync(0xffffffffu, mbar_wait(sum_full, 0));
        ok = __all_sync(0xffffffffu, ok && have_sum && !*failed && (tiles == 0 || mbar_wait(mma_done, 0)));
        if (ok) {
            tc_fence_after();
            float o[kDtcN];
            if (tiles > 0) {
                tmem_ld16_nowait(lane_base + kDtcOCol, o, 0);
                tmem_wait_regs(o);
            }
            const int d = row;  // this thread's O^T row
#pragma unroll
            for (int h = 0; h < kDtcGroups; ++h) {
                const float l = ((lsum[h] + lsum[kDtcN + h]) + (lsum[2 * kDtcN + h] + lsum[3 * kDtcN + h]));
                const float ov = tiles > 0 ? __fadd_rn(o[h], o[kDtcGroups + h]) : 0.f;  // P hi + P lo parts
                const int qh = kvh * kDtcGroups + h;
                if (a.splits == 1) {
                    if (ctx > 0) a.out[b * a.out_stride + static_cast<long long>(qh) * kDtcDim + d] = ov * __fdiv_rn(1.0f, l);
                } else {
                    float* part = a.partials +
                                  (((static_cast<long long>(b) * a.kv_heads + kvh) * a.splits + split) * kDtcGroups + h) *
                                      kPartialStride;
                    part[d] = ov;
                    if (d == 0) {
                        // natural-log reference: p = exp(s * scale - (m_ref - 8) ln 2)
                        part[kDtcDim] = m_ref[h] == -INFINITY ? 0.f : (m_ref[h] - kPtcOffset) * 0.6931471805599453f;
                        part[kDtcDim + 1] = tiles > 0 ? l : 0.f;
                    }
                }
            }
        } else if (lane == 0) {
            *failed = 1;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kDtcKWarp) {
        mbar_wait(mma_done, 0);
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kDtcTmemCols)
                     : "memory");
    }
}

bool batch_tc_supported(int kv_dtype, int head_dim, int groups) {
    return kv_dtype == 1 && head_dim == kDtcDim && groups == kDtcGroups && tensor_map_encoder() != nullptr;
}

// One layer's caches of every sequence ([batch][layers][kv_heads][capacity]
// [128] fp16, this layer's slice at `base`) as a 4-D map (d, time, kv head,
// sequence) with a [1][1][128][64] box; keys past the capacity read as zeros.
static bool batch_cache_map(CUtensorMap* out, const void* base, int kv_heads, int batch, int capacity,
                            long long batch_stride) {
    auto encode = tensor_map_encoder();
    if (!encode) return false;
    const cuuint64_t dims[4] = {static_cast<cuuint64_t>(kDtcDim), static_cast<cuuint64_t>(capacity),
                                static_cast<cuuint64_t>(kv_heads), static_cast<cuuint64_t>(batch)};
    const cuuint64_t strides[3] = {kDtcDim * 2ull, static_cast<cuuint64_t>(capacity) * kDtcDim * 2ull,
                                   static_cast<cuuint64_t>(batch_stride) * 2ull};
    const cuuint32_t box[4] = {kDtcDim / 2, kDtcKeys, 1, 1};
    const cuuint32_t elem[4] = {1, 1, 1, 1};
    return encode(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Batched decode attention of layer l on the tensor cores: q/k norm, RoPE
// and the K/V append by the prefill's rope kernel (one row per sequence),
// then decode_attention_tc_kernel, then the split merge.
int launch_batch_attention_tc(const h4b_model* m, const h4b_batch_state* s, int l, cudaStream_t stream) {
    static std::atomic<bool> opted_in[kMaxDevices];
    int dev = 0;
    H4B_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return H4B_EUNSUPPORTED;
    if (!opted_in[dev].load(std::memory_order_acquire)) {
        H4B_CUDA_TRY(cudaFuncSetAttribute(decode_attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          kDtcSmem));
        opted_in[dev].store(true, std::memory_order_release);
    }
    const int B = s->batch, d = m->head_dim;
    const int q_size = m->heads * d, kv_size = m->kv_heads * d, qkv_rows = q_size + 2 * kv_size;
    const size_t kv_layer = static_cast<size_t>(m->kv_heads) * s->capacity * d;  // elements
    const long long batch_stride = static_cast<long long>(m->layers) * static_cast<long long>(kv_layer);
    __half* kc = static_cast<__half*>(s->k_cache) + l * kv_layer;
    __half* vc = static_cast<__half*>(s->v_cache) + l * kv_layer;
    const long long pairs = static_cast<long long>(B) * (m->heads + m->kv_heads);
    prefill_rope_append_kernel<__half><<<static_cast<int>((pairs + kRopeWarps - 1) / kRopeWarps), 32 * kRopeWarps, 0,
                                         stream>>>(
        s->qkv, qkv_rows, m->heads, m->kv_heads, m->norm_q + static_cast<size_t>(l) * d,
        m->norm_k + static_cast<size_t>(l) * d, m->rope_cos, m->rope_sin, m->eps, s->positions, B, kc, vc,
        static_cast<long long>(s->capacity) * d, d, s->capacity, batch_stride);
    H4B_CUDA_TRY(cudaGetLastError());
    CUtensorMap kmap, vmap;
    if (!batch_cache_map(&kmap, kc, m->kv_heads, B, s->capacity, batch_stride) ||
        !batch_cache_map(&vmap, vc, m->kv_heads, B, s->capacity, batch_stride))
        return H4B_EUNSUPPORTED;
    // splits: one wave of CTAs (one fits per SM) when the batch's (sequence,
    // kv head) pairs leave at least half the SMs idle, else about two CTAs per
    // SM; at most the state's count (its partials are sized for that);
    // whole-sequence CTAs when the batch alone fills the GPU
    const int units = B * m->kv_heads;
    const int splits =
        std::max(1, std::min(s->attn_splits, 2 * units <= sm_count() ? sm_count() / units
                                                                       : (2 * sm_count() + units - 1) / units));
    const DtcArgs a{s->qkv, qkv_rows, s->positions, splits, m->kv_heads, s->capacity, s->attn_partials, s->attended,
                    q_size};
    decode_attention_tc_kernel<<<dim3(splits, m->kv_heads, B), kDtcThreads, kDtcSmem, stream>>>(kmap, vmap, a);
    H4B_CUDA_TRY(cudaGetLastError());
    if (splits > 1) {
        AttnArgs ma = {};
        ma.partials = s->attn_partials;
        ma.out = s->attended;
        ma.out_batch_stride = q_size;
        ma.splits = splits;
        ma.groups = kDtcGroups;
        ma.kv_heads = m->kv_heads;
        gqa_merge_kernel<<<dim3(1, m->kv_heads, B), 32 * kDtcGroups, 0, stream>>>(ma);
        H4B_CUDA_TRY(cudaGetLastError());
    }
    return 0;
}

}  // namespace h4b
