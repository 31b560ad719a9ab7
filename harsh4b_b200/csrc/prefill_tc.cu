// Prefill attention on the 5th-generation tensor cores: tcgen05.mma
// kind::f16 with fp32 accumulators in tensor memory, K/V tiles fed by TMA.
//
// Scope: an fp16 K/V cache, head_dim 128 and 4 q heads per kv head (the
// Qwen3-4B shape); other shapes take the fp32 kernels in prefill.cu.
//
// Work split: one CTA per (kv head, block of 32 prompt positions). Its 128
// query rows are (q head h of the kv head's group, position q0 + i), row
// r = 32 h + i, so the four heads that share a K/V tile share one MMA. Keys
// advance 64 per tile over [0, last position of the block]; each row masks
// the keys past its own position (causal).
//
// Precision: this path meets a tolerance, not the decode's bit order. The
// fp16 K and V are the cache's own values, exact as MMA operands. q and the
// probabilities p are fp32 and enter as two fp16 terms each, hi = fp16(x)
// and lo = fp16(x - hi), so q.k and p.v are each the sum of two MMAs with
// fp32 accumulation: about 2^-22 relative representation error instead of
// fp16's 2^-11. The softmax runs in base 2 (scores times log2(e)/sqrt(d))
// with the running maximum lowered by 8, so p <= 2^8 (an exact power-of-two
// scale that cancels in o / l) keeps the lo terms clear of fp16 subnormals.
//
// Operands: q (hi, lo) and the probability tiles P (hi, lo) live in tensor
// memory, the A operands of the MMAs (row = lane, two fp16 per 32-bit
// column); only the K and V tiles are read from shared memory. A tile's P is
// written over its own S columns once the row warps hold S in registers.
//
// Warps: 0-3 are the row warps (thread = query row; TMEM lane quarter =
// warp), 4 loads K tiles and owns the tensor memory, 5 loads V tiles, 6
// issues the MMAs (one elected thread). Per key tile j (128 keys), with the
// score accumulator S (and P over it) double-buffered (b = j % 2), K and V in
// kStages stages and one output accumulator O in tensor memory:
//   MMA:   S[b] = Qhi K_j^T + Qlo K_j^T                  -> s_full[b], k_empty
//   rows:  load S[b]; masked maximum, p; P[b] = (phi, plo) over S[b]
//                                                         -> p_full[b]
//   MMA:   O += Phi V_j + Plo V_j                        -> o_full, v_empty
// The MMA thread issues P.V for tile j, then S for tile j + 2 into the same
// columns: the tensor cores run a CTA's MMAs in issue order, so the P.V has
// read P before the S overwrites it; and s_full for tile j also stands for
// the completion of P.V j - 2 (a commit tracks every earlier MMA of its
// thread). The tile is 128 keys so that each MMA does more work: the MMA
// thread's issue of the many small MMAs of 64-key tiles was the bound.
// O is scaled lazily: each row keeps a reference maximum m_ref and forms
// p = 2^(s - m_ref + 8); only when a tile's maximum passes m_ref + 7 (p would
// leave fp16's range) does the row move m_ref up, and the warp then rescales
// its O rows in tensor memory (after the P.V MMAs issued so far completed)
// before publishing the tile's P. The result, o / l, is the same quotient.
//
// Every wait is bounded (mbar_wait). A role whose wait runs out reports
// kStatusWaitTimeout, marks the CTA as failed and stops; the producers wait
// for the copies they issued, the MMA thread commits a last barrier that the
// tensor-memory owner waits on, and the tensor memory is freed on every path.

namespace h4b {

constexpr int kPtcPositions = 32;                          // prompt positions per CTA
constexpr int kPtcGroups = 4;                              // q heads per kv head
constexpr int kPtcRows = kPtcPositions * kPtcGroups;       // MMA M = 128
constexpr int kPtcKeys = 128;                              // keys per tile (the S MMA's N)
constexpr int kPtcDim = 128;                               // head_dim (the P.V MMA's N)
constexpr int kPtcStages = 3;                              // K and V tile stages
constexpr int kPtcRowWarps = 4, kPtcKWarp = 4, kPtcVWarp = 5, kPtcMmaWarp = 6;
constexpr int kPtcThreads = 32 * 7;

// Shared memory, every tile 1024-byte aligned (the 128-byte swizzle atom):
//   K: [stage][d half][128 keys x 128 B]                  kPtcStages x 32 KB
//   V: [stage][d half][128 keys x 128 B]                  kPtcStages x 32 KB
constexpr int kPtcHalfTile = kPtcKeys * 128;               // 16 KB: 128 keys x 64 dims of fp16
constexpr int kPtcKOff = 0;
constexpr int kPtcVOff = kPtcKOff + kPtcStages * 2 * kPtcHalfTile;
constexpr int kPtcBarOff = kPtcVOff + kPtcStages * 2 * kPtcHalfTile;
constexpr int kPtcBarBytes = 256;
constexpr int kPtcSmem = kPtcBarOff + kPtcBarBytes + 1024;  // + alignment slack
static_assert(kPtcSmem <= 232448, "shared memory per CTA");
static_assert((4 * kPtcStages + 7) * 8 + 8 <= kPtcBarBytes, "barrier area");

// Tensor memory columns (32-bit): q hi, q lo (64 each: 128 fp16), S[0], S[1]
// (128 fp32 each; P[b] over S[b]: hi then lo, 64 columns each = 128 fp16),
// O (128 fp32).
constexpr uint32_t kPtcTmemCols = 512;
constexpr uint32_t kPtcQCol = 0, kPtcSCol = 128, kPtcOCol = 384;
// Lazy rescaling: p = 2^(s - m_ref + kPtcOffset), m_ref moves when a score
// passes m_ref + kPtcSlack, so p < 2^(kPtcOffset + kPtcSlack) = 2^15 < fp16 max.
constexpr float kPtcOffset = 8.f, kPtcSlack = 7.f;

// Instruction descriptors (kind::f16): D f32 (bits 4-5 = 1), A and B f16
// (format 0), N >> 3 at bit 17, M >> 4 at bit 24; P.V reads B (the V tile)
// MN-major (bit 16), S reads both operands K-major.
constexpr uint32_t kPtcIdescS = (1u << 4) | (static_cast<uint32_t>(kPtcKeys >> 3) << 17) |
                                (static_cast<uint32_t>(kPtcRows >> 4) << 24);
constexpr uint32_t kPtcIdescPV = (1u << 4) | (1u << 16) | (static_cast<uint32_t>(kPtcDim >> 3) << 17) |
                                 (static_cast<uint32_t>(kPtcRows >> 4) << 24);

// Shared-memory descriptor of an MN-major operand in the 128-byte swizzle
// layout: 64 fp16 of the N dimension per 128-byte row, 8-row groups of the
// K dimension 1024 bytes apart (stride byte offset), the next 64 of N
// `mn_stride` bytes on (leading byte offset); version 1, SWIZZLE_128B.
__device__ __forceinline__ uint64_t sw128_mn_desc(const void* tile, uint32_t mn_stride) {
    return static_cast<uint64_t>((smem_addr(tile) >> 4) & 0x3FFF) |
           (static_cast<uint64_t>((mn_stride >> 4) & 0x3FFF) << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void tc_mma_f16(uint32_t tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// The same with A in tensor memory (K-major: row = lane, two fp16 per column).
__device__ __forceinline__ void tc_mma_f16_ts(uint32_t tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(tmem), "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];"
        ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
        : "memory");
}

// 16 columns of this warp's TMEM lane quarter into v[off .. off + 15],
// without the wait: the caller issues several, then tmem_wait_regs.
template <int N>
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, float (&v)[N], int off) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=f"(v[off + 0]), "=f"(v[off + 1]), "=f"(v[off + 2]), "=f"(v[off + 3]), "=f"(v[off + 4]),
          "=f"(v[off + 5]), "=f"(v[off + 6]), "=f"(v[off + 7]), "=f"(v[off + 8]), "=f"(v[off + 9]),
          "=f"(v[off + 10]), "=f"(v[off + 11]), "=f"(v[off + 12]), "=f"(v[off + 13]), "=f"(v[off + 14]),
          "=f"(v[off + 15])
        : "r"(taddr));
}

// tcgen05.wait::ld with the loaded registers as operands, so no use of them
// is scheduled before the wait.
template <int N>
__device__ __forceinline__ void tmem_wait_regs(float (&v)[N]) {
    static_assert(N % 16 == 0, "groups of 16");
#pragma unroll
    for (int g = 0; g < N; g += 16)
        asm volatile("tcgen05.wait::ld.sync.aligned;"
                     : "+f"(v[g + 0]), "+f"(v[g + 1]), "+f"(v[g + 2]), "+f"(v[g + 3]), "+f"(v[g + 4]),
                       "+f"(v[g + 5]), "+f"(v[g + 6]), "+f"(v[g + 7]), "+f"(v[g + 8]), "+f"(v[g + 9]),
                       "+f"(v[g + 10]), "+f"(v[g + 11]), "+f"(v[g + 12]), "+f"(v[g + 13]), "+f"(v[g + 14]),
                       "+f"(v[g + 15])
                     :
                     : "memory");
}

// 16 columns of this warp's TMEM lane quarter from v[off .. off + 15].
template <int N>
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[N], int off) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        ::"r"(taddr), "f"(v[off + 0]), "f"(v[off + 1]), "f"(v[off + 2]), "f"(v[off + 3]), "f"(v[off + 4]),
          "f"(v[off + 5]), "f"(v[off + 6]), "f"(v[off + 7]), "f"(v[off + 8]), "f"(v[off + 9]), "f"(v[off + 10]),
          "f"(v[off + 11]), "f"(v[off + 12]), "f"(v[off + 13]), "f"(v[off + 14]), "f"(v[off + 15])
        : "memory");
}

template <int N>
__device__ __forceinline__ void tmem_st16u(uint32_t taddr, const uint32_t (&v)[N], int off) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        ::"r"(taddr), "r"(v[off + 0]), "r"(v[off + 1]), "r"(v[off + 2]), "r"(v[off + 3]), "r"(v[off + 4]),
          "r"(v[off + 5]), "r"(v[off + 6]), "r"(v[off + 7]), "r"(v[off + 8]), "r"(v[off + 9]), "r"(v[off + 10]),
          "r"(v[off + 11]), "r"(v[off + 12]), "r"(v[off + 13]), "r"(v[off + 14]), "r"(v[off + 15])
        : "memory");
}

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// fp32 -> (hi, lo) fp16 terms, packed two values per 32-bit word.
__device__ __forceinline__ void split_pair(float a, float b, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(a, b);
    const float2 back = __half22float2(h);
    const __half2 l = __floats2half2_rn(a - back.x, b - back.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}

__global__ void __launch_bounds__(kPtcThreads, 1)
    prefill_attention_tc_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                                const float* qkv, int qkv_stride, const int32_t* positions, int count, float* out,
                                int out_stride) {
    extern __shared__ uint8_t ptc_smem_raw[];
    uint8_t* smem = ptc_smem_raw + ((1024u - (smem_addr(ptc_smem_raw) & 1023u)) & 1023u);
    uint64_t* k_full = reinterpret_cast<uint64_t*>(smem + kPtcBarOff);
    uint64_t* k_empty = k_full + kPtcStages;
    uint64_t* v_full = k_empty + kPtcStages;
    uint64_t* v_empty = v_full + kPtcStages;
    uint64_t* s_full = v_empty + kPtcStages;  // [2]
    uint64_t* p_full = s_full + 2;             // [2]
    uint64_t* o_full = p_full + 2;             // one phase per P.V tile
    uint64_t* q_ready = o_full + 1;
    uint64_t* mma_done = q_ready + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
    volatile int* failed = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // the longest contexts (the last position blocks) first, so the tail is short
    const int kvh = blockIdx.x, q0 = (gridDim.y - 1 - blockIdx.y) * kPtcPositions;
    const int nq = min(kPtcPositions, count - q0);
    int max_ctx = 0;  // keys [0, max_ctx) are read by some row of the block
    for (int i = 0; i < nq; ++i) max_ctx = max(max_ctx, positions[q0 + i] + 1);
    const int tiles = (max_ctx + kPtcKeys - 1) / kPtcKeys;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kPtcStages; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&s_full[b], 1);
            mbar_init(&p_full[b], kPtcRowWarps);
        }
        mbar_init(o_full, 1);
        mbar_init(q_ready, kPtcRowWarps);
        mbar_init(mma_done, 1);
        *failed = wait_failed_before() ? 1 : 0;
        fence_mbar_init();
    }
    if (warp == kPtcKWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_addr(tmem_slot)), "r"(kPtcTmemCols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    auto k_half = [&](int s, int half) { return smem + kPtcKOff + (s * 2 + half) * kPtcHalfTile; };
    auto v_half = [&](int s, int half) { return smem + kPtcVOff + (s * 2 + half) * kPtcHalfTile; };

    // Each waiter below meets every phase of the barriers it waits on in
    // order, at most one phase behind (see the row warps' V tail wait).
    if (warp == kPtcKWarp || warp == kPtcVWarp) {
        if (lane == 0) {  // TMA producer of the K (or V) tiles
            const bool is_k = warp == kPtcKWarp;
            const CUtensorMap* map = is_k ? &kmap : &vmap;
            uint64_t* full = is_k ? k_full : v_full;
            uint64_t* empty = is_k ? k_empty : v_empty;
            int issued = 0;
            if (!*failed) {
                asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
                for (int j = 0; j < tiles; ++j) {
                    const int s = j % kPtcStages;
                    if (*failed) break;
                    if (j >= kPtcStages && !mbar_wait(&empty[s], (j / kPtcStages - 1) & 1)) {
                        *failed = 1;
                        break;
                    }
                    uint8_t* dst0 = is_k ? k_half(s, 0) : v_half(s, 0);
                    uint8_t* dst1 = is_k ? k_half(s, 1) : v_half(s, 1);
                    mbar_arrive_expect_tx(&full[s], 2 * kPtcHalfTile);
                    tma_load_3d(dst0, map, 0, j * kPtcKeys, kvh, &full[s]);
                    tma_load_3d(dst1, map, kPtcDim / 2, j * kPtcKeys, kvh, &full[s]);
                    issued = j + 1;
                }
            }
            // the copies issued must land before the CTA may exit
            for (int j = issued > kPtcStages ? issued - kPtcStages : 0; j < issued; ++j)
                mbar_wait(&full[j % kPtcStages], (j / kPtcStages) & 1);
        }
    } else if (warp == kPtcMmaWarp) {
        if (lane == 0) {  // MMA issuer
            auto issue_s = [&](int j) -> bool {
                const int s = j % kPtcStages, b = j & 1;
                if (*failed) return false;
                if (!mbar_wait(&k_full[s], (j / kPtcStages) & 1)) return false;
                tc_fence_after();
#pragma unroll
                for (int part = 0; part < 2; ++part)
#pragma unroll
                    for (int kk = 0; kk < kPtcDim / 16; ++kk) {
                        // A: 16 dims = 8 columns of q; B: 16 dims = 32 bytes = +2 in the address field
                        const uint32_t a = tmem + kPtcQCol + 64 * part + 8 * kk;
                        const uint64_t bd = sw128_desc(k_half(s, kk >> 2)) + 2 * (kk & 3);
                        tc_mma_f16_ts(tmem + kPtcSCol + b * kPtcKeys, a, bd, kPtcIdescS, (part | kk) != 0);
                    }
                tc_commit(&k_empty[s]);
                tc_commit(&s_full[b]);
                return true;
            };
            auto issue_pv = [&](int j) -> bool {
                const int s = j % kPtcStages, b = j & 1;
                if (*failed) return false;
                if (!mbar_wait(&p_full[b], (j >> 1) & 1)) return false;
                if (!mbar_wait(&v_full[s], (j / kPtcStages) & 1)) return false;
                tc_fence_after();
#pragma unroll
                for (int part = 0; part < 2; ++part)
#pragma unroll
                    for (int kk = 0; kk < kPtcKeys / 16; ++kk) {
                        // A: 16 keys = 8 columns of P; B: 16 keys = 2 groups of 8 rows = 2048 bytes
                        const uint32_t a = tmem + kPtcSCol + kPtcKeys * b + 64 * part + 8 * kk;
                        const uint64_t bd = sw128_mn_desc(v_half(s, 0) + kk * 2048, kPtcHalfTile);
                        tc_mma_f16_ts(tmem + kPtcOCol, a, bd, kPtcIdescPV, (j | part | kk) != 0);
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
            tc_commit(mma_done);  // arrives once every MMA issued above has completed
        }
    } else {  // row warps: thread = query row r = 32 h + i
        const int h = warp, i = lane;  // query row 32 h + i = this thread's TMEM lane
        const bool valid = i < nq;
        const int pos = valid ? positions[q0 + i] : -1;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(32 * h) << 16);
        {
            const float* qrow = qkv + static_cast<long long>(q0 + (valid ? i : 0)) * qkv_stride +
                                static_cast<long long>(kvh * kPtcGroups + h) * kPtcDim;
#pragma unroll 1
            for (int c0 = 0; c0 < kPtcDim; c0 += 32) {  // 32 dims = 16 columns per part
                uint32_t hi[16], lo[16];
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (valid) x = reinterpret_cast<const float4*>(qrow + c0)[c];
                    split_pair(x.x, x.y, hi[2 * c], lo[2 * c]);
                    split_pair(x.z, x.w, hi[2 * c + 1], lo[2 * c + 1]);
                }
                tmem_st16u(lane_base + kPtcQCol + c0 / 2, hi, 0);
                tmem_st16u(lane_base + kPtcQCol + 64 + c0 / 2, lo, 0);
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(q_ready);

        // log2(e) / sqrt(128): scores in base-2 units
        const float score_scale = 1.4426950408889634f * 0.08838834764831845f;
        float m_ref = -INFINITY, l = 0.f;
        bool ok = true;

        for (int j = 0; j < tiles && ok; ++j) {
            const int b = j & 1;
            ok = __all_sync(0xffffffffu, !*failed && mbar_wait(&s_full[b], (j >> 1) & 1));
            if (!ok) break;
            tc_fence_after();
            float sv[kPtcKeys];
#pragma unroll
            for (int c0 = 0; c0 < kPtcKeys; c0 += 16) tmem_ld16_nowait(lane_base + kPtcSCol + b * kPtcKeys + c0, sv, c0);
            tmem_wait_regs(sv);

            // causal mask (only tiles that reach past some row's position) and
            // the tile maximum, in raw q.k units (the scale is positive)
            const int kbase = j * kPtcKeys;
            if (!__all_sync(0xffffffffu, kbase + kPtcKeys - 1 <= pos)) {
#pragma unroll
                for (int c = 0; c < kPtcKeys; ++c) sv[c] = kbase + c <= pos ? sv[c] : -INFINITY;
            }
            // pairwise (the maximum is order-free; a tree keeps the dependent
            // chain at log2(64) steps instead of 63)
            float tm[kPtcKeys / 2];
#pragma unroll
            for (int c = 0; c < kPtcKeys / 2; ++c) tm[c] = fmaxf(sv[c], sv[c + kPtcKeys / 2]);
#pragma unroll
            for (int w = kPtcKeys / 4; w >= 1; w >>= 1)
#pragma unroll
                for (int c = 0; c < w; ++c) tm[c] = fmaxf(tm[c], tm[c + w]);
            const float mx = tm[0];
            const float tmax = mx * score_scale;  // -inf stays -inf
            const bool move = tmax > m_ref + kPtcSlack;
            const bool rescale = move && m_ref != -INFINITY;
            if (__any_sync(0xffffffffu, rescale)) {
                // O (every P.V issued so far: tiles < j) times 2^(m_ref - tmax)
                ok = __all_sync(0xffffffffu, !*failed && mbar_wait(o_full, (j - 1) & 1));
                if (!ok) break;
                tc_fence_after();
                const float alpha = rescale ? ex2_approx(m_ref - tmax) : 1.f;
#pragma unroll
                for (int c0 = 0; c0 < kPtcDim; c0 += 32) {
                    float v[32];
                    tmem_ld16_nowait(lane_base + kPtcOCol + c0, v, 0);
                    tmem_ld16_nowait(lane_base + kPtcOCol + c0 + 16, v, 16);
                    tmem_wait_regs(v);
#pragma unroll
                    for (int k = 0; k < 32; ++k) v[k] *= alpha;
                    tmem_st16(lane_base + kPtcOCol + c0, v, 0);
                    tmem_st16(lane_base + kPtcOCol + c0 + 16, v, 16);
                }
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                l *= alpha;
            }
            if (move) m_ref = tmax;
            // p = 2^(s * scale - (m_ref - offset)); masked keys give 2^-inf = 0
            const float nbase = m_ref == -INFINITY ? 0.f : kPtcOffset - m_ref;
            // eight partial sums (one per key of a 16-byte chunk): short
            // dependent chains for the row sum
            float part[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) part[k] = 0.f;
#pragma unroll
            for (int c0 = 0; c0 < kPtcKeys; c0 += 32) {  // 32 keys = 16 columns per part
                uint32_t hi[16], lo[16];
#pragma unroll
                for (int c = 0; c < 32; c += 8) {
                    float pv[8];
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        pv[k] = ex2_approx(__fmaf_rn(sv[c0 + c + k], score_scale, nbase));
                        part[k] += pv[k];
                    }
#pragma unroll
                    for (int k = 0; k < 8; k += 2) split_pair(pv[k], pv[k + 1], hi[(c + k) / 2], lo[(c + k) / 2]);
                }
                tmem_st16u(lane_base + kPtcSCol + kPtcKeys * b + c0 / 2, hi, 0);
                tmem_st16u(lane_base + kPtcSCol + kPtcKeys * b + 64 + c0 / 2, lo, 0);
            }
            l += ((part[0] + part[4]) + (part[2] + part[6])) + ((part[1] + part[5]) + (part[3] + part[7]));
            if (j == tiles - 1 && max_ctx < kbase + kPtcKeys) {
                // Keys [max_ctx, tile end) get p = 0 from every row, but their V
                // rows (cache entries past the context, or the TMA's zero fill
                // past the capacity) must not be NaN: 0 * NaN would reach the
                // sum. Zero them once the tile has landed; each row warp zeroes
                // its own share before its p_full arrival, and the P.V MMAs
                // wait for all four. s_full for this tile stood for the
                // completion of P.V j - 2, so v_full's current phase is this
                // tile's.
                const int s = j % kPtcStages;
                ok = __all_sync(0xffffffffu, !*failed && mbar_wait(&v_full[s], (j / kPtcStages) & 1));
                if (!ok) break;
                const int first = max_ctx - kbase;
                const int chunks = (kPtcKeys - first) * 8;  // 16-byte chunks per d half
                for (int t = threadIdx.x; t < 2 * chunks; t += 32 * kPtcRowWarps) {
                    const int half = t / chunks, idx = t % chunks;
                    *reinterpret_cast<uint4*>(v_half(s, half) + (first + idx / 8) * 128 + (idx % 8) * 16) =
                        make_uint4(0u, 0u, 0u, 0u);
                }
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");  // P (and any O rescale) written
            fence_proxy_async_smem();  // the zeroed V rows -> visible to the tensor cores
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[b]);
        }
        // every MMA complete (the last commit of the MMA thread): O is final
        ok = __all_sync(0xffffffffu, ok && tiles > 0 && !*failed && mbar_wait(mma_done, 0));
        if (ok) {
            tc_fence_after();
            const float inv = __fdiv_rn(1.0f, l);
            float* orow = out + static_cast<long long>(q0 + (valid ? i : 0)) * out_stride +
                          static_cast<long long>(kvh * kPtcGroups + h) * kPtcDim;
#pragma unroll
            for (int c0 = 0; c0 < kPtcDim; c0 += 32) {
                float v[32];
                tmem_ld16_nowait(lane_base + kPtcOCol + c0, v, 0);
                tmem_ld16_nowait(lane_base + kPtcOCol + c0 + 16, v, 16);
                tmem_wait_regs(v);
                if (valid && pos >= 0) {
#pragma unroll
                    for (int c = 0; c < 32; c += 4)
                        *reinterpret_cast<float4*>(orow + c0 + c) =
                            make_float4(v[c] * inv, v[c + 1] * inv, v[c + 2] * inv, v[c + 3] * inv);
                }
            }
        } else if (tiles > 0 && lane == 0) {
            *failed = 1;
        }
        ok = ok || tiles == 0;
        if (!ok && lane == 0) *failed = 1;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kPtcKWarp) {
        // the MMAs must be complete before their tensor memory is released
        mbar_wait(mma_done, 0);
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPtcTmemCols)
                     : "memory");
    }
}

// The layer's K (or V) cache [kv_heads][capacity][128] fp16 as a 3-D tensor
// map with a [1][64][64] box (128-byte rows, 128-byte swizzle); keys past the
// capacity read as zeros.
static bool kv_cache_map(CUtensorMap* out, const void* base, int kv_heads, int capacity) {
    auto encode = tensor_map_encoder();
    if (!encode) return false;
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kPtcDim), static_cast<cuuint64_t>(capacity),
                                static_cast<cuuint64_t>(kv_heads)};
    const cuuint64_t strides[2] = {kPtcDim * 2ull, static_cast<cuuint64_t>(capacity) * kPtcDim * 2ull};
    const cuuint32_t box[3] = {kPtcDim / 2, kPtcKeys, 1};
    const cuuint32_t elem[3] = {1, 1, 1};
    return encode(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool prefill_tc_supported(int kv_dtype, int head_dim, int groups) {
    return kv_dtype == 1 && head_dim == kPtcDim && groups == kPtcGroups && tensor_map_encoder() != nullptr;
}

// Attention of `count` prompt rows (q in qkv, already normalised and
// rotated; K/V already appended) into `out`, for one layer's fp16 cache.
int launch_prefill_attention_tc(const float* qkv, int qkv_stride, const __half* kcache, const __half* vcache,
                                int kv_heads, int capacity, const int32_t* positions, int count, float* out,
                                int out_stride, cudaStream_t stream) {
    static std::atomic<bool> opted_in[kMaxDevices];
    int dev = 0;
    H4B_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return H4B_EUNSUPPORTED;
    if (!opted_in[dev].load(std::memory_order_acquire)) {
        H4B_CUDA_TRY(cudaFuncSetAttribute(prefill_attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          kPtcSmem));
        opted_in[dev].store(true, std::memory_order_release);
    }
    if ((reinterpret_cast<uintptr_t>(kcache) & 15) || (reinterpret_cast<uintptr_t>(vcache) & 15) ||
        (reinterpret_cast<uintptr_t>(qkv) & 15) || (reinterpret_cast<uintptr_t>(out) & 15) || (qkv_stride & 3) ||
        (out_stride & 3))
        return H4B_EINVAL;
    CUtensorMap kmap, vmap;
    if (!kv_cache_map(&kmap, kcache, kv_heads, capacity) || !kv_cache_map(&vmap, vcache, kv_heads, capacity))
        return H4B_EUNSUPPORTED;
    const dim3 grid(kv_heads, (count + kPtcPositions - 1) / kPtcPositions);
    prefill_attention_tc_kernel<<<grid, kPtcThreads, kPtcSmem, stream>>>(kmap, vmap, qkv, qkv_stride, positions,
                                                                         count, out, out_stride);
    H4B_CUDA_TRY(cudaGetLastError());
    return 0;
}

}  // namespace h4b
