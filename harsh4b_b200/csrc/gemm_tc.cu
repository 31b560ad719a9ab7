// Batched int4 x int8 GEMM on the 5th-generation tensor cores (tcgen05 with
// the accumulator in tensor memory), fed by TMA:
//   out[m][n] = float(sum_k w[n][k] * x[m][k]) * act_scale[m] * w_scale[n]
// the same contract and result bits as gemm.cu (integer sums are exact).
//
// Tile: 128 weight rows (the MMA's M) x TOK tokens (its N: 64, 128 or 256),
// K advancing 128 per pipeline stage. A CTA has 4 G + 2 warps (G unpack
// groups: 5 at TOK 256, else 4):
//   warp 4 G lane 0: TMA producer -- per stage, the packed weight tile
//           (128 rows x 64 bytes, 64-byte swizzle) and the activation tile
//           (TOK rows x 128 bytes, 128-byte swizzle) land on the stage's
//           `full` mbarrier; the warp also allocates and frees the tensor
//           memory. Shared memory holds only this ring (5 stages at TOK
//           256, else 8: one per unpacked tile);
//   warps 0 .. 4 G - 1: unpack groups of four warps, group g taking stages
//           g, g + G, ...: thread = weight row (its warp's TMEM lane quarter),
//           it reads the row's 64 packed bytes, expands them to 128 signed
//           int8 codes and stores them with tcgen05.st into one of the
//           group's unpacked tiles in tensor memory (32 columns, four codes
//           per column; two tiles per group used in turn below TOK 256) --
//           the MMA's A operand (tile s for stage s) -- then arrives on the
//           tile's `aready`. After
//           the last stage the first sixteen warps are the epilogue, warp w
//           reading TMEM lane quarter w % 4 (32 rows) for column slice w / 4;
//   warp 4 G + 1 lane 0: issues tcgen05.mma kind::i8 (A s8 weights from
//           tensor memory, B s8 activations from shared memory, D s32 in
//           TMEM), 4 per stage (K = 32 each), and tcgen05.commit to the
//           stage's `empty`, which frees the stage and its tile (the MMA
//           thread waits only on `aready`: its group saw the stage land before
//           arriving); a final commit signals
//           the epilogue.
// Every wait is bounded (mbar_wait). A role whose wait runs out reports
// kStatusWaitTimeout, marks the CTA as failed and stops issuing; the
// producer still waits for the copies it issued, the MMA thread still
// commits (so the epilogue's wait ends once its MMAs are done), and the
// tensor memory is freed on every path.
#include <cuda.h>
#include <cudaTypedefs.h>

namespace h4b {

constexpr int kTcRows = 128;     // weight rows per CTA (MMA M)
constexpr int kTcK = 128;        // k per stage: one 128-byte swizzle atom of int8
constexpr int kTcGroupWarps = 4;  // an unpack group: one warp per TMEM lane quarter

template <int TOK>
struct TcCfg {
    // Unpack groups: group g owns the k-steps g, g + kGroups, ... and with
    // them the TMA stages and unpacked tiles g, g + kGroups, ... (the stage
    // count is a multiple of the groups, so a group always revisits its own
    // stages round by round).
    static constexpr int kGroups = TOK == 256 ? 5 : 4;
    // Unpacked weight tiles in tensor memory: two per group below TOK 256, so
    // a group expands its next stage while the MMAs still read its previous
    // one (each tile is free again only when the MMA thread's commit lands);
    // one per group at TOK 256, whose accumulator takes 256 columns.
    static constexpr int kSlotsPerGroup = TOK == 256 ? 1 : 2;
    static constexpr int kASlots = kGroups * kSlotsPerGroup;
    // One TMA stage per unpacked tile: stage s and tile s are used by the
    // same iterations, so a single commit per stage frees both.
    static constexpr int kStages = TOK == 256 ? 5 : 8;
    static constexpr int kUnpackWarps = kGroups * kTcGroupWarps;
    static constexpr int kProducerWarp = kUnpackWarps, kMmaWarp = kUnpackWarps + 1;
    static constexpr int kThreads = 32 * (kUnpackWarps + 2);
    static constexpr int kBBytes = TOK * kTcK;               // activations, int8
    static constexpr int kPackedBytes = kTcRows * kTcK / 2;  // packed weights
    static constexpr int kBOff = 0, kPackedOff = kBBytes;    // inside a TMA stage
    static constexpr int kStageBytes = kBBytes + kPackedBytes;
    static constexpr int kBarrierOff = kStages * kStageBytes;
    static constexpr int kBarrierBytes = 512;
    static constexpr int kSmem = kBarrierOff + kBarrierBytes + 1024;  // + alignment slack
    // tensor memory: the accumulator (TOK columns; at TOK 64 two of them, one
    // per row tile of a stream-K range), then the unpacked weight tiles
    // (128 rows x 128 int8 = 32 columns each)
    static constexpr int kAccs = TOK == 64 ? 2 : 1;
    static constexpr uint32_t kACol = kAccs * TOK;
    static constexpr uint32_t kTmemCols = kACol + 32 * kASlots <= 256 ? 256 : 512;
    static_assert(kStageBytes % 1024 == 0, "tiles keep the 1024-byte swizzle alignment");
    static_assert(kStages % kGroups == 0, "each group must own whole stages");
    static_assert(kStages == kGroups * kSlotsPerGroup, "stage s is unpacked into tile s");
    static_assert(kSmem <= 232448, "shared memory per CTA");
    static_assert(kACol + 32 * kASlots <= kTmemCols, "tensor memory");
    static_assert(2 * kStages * 8 + kASlots * 8 + 16 <= kBarrierBytes, "barrier area");
};

struct TcArgs {
    const float* act_scale;  // [M]
    const float* w_scale;    // [N]
    float* out;              // [M][N]
    int M, N, K;
    int32_t* out_i32;        // when set: the exact int32 sums [M][N] instead of `out`
    int32_t* split_acc;      // split-K (gridDim.z > 1): K slices add their int32 sums here
    int residual;            // out[m][n] = out[m][n] + value instead of value
    // stream-K (M <= TOK = 64, split_acc set): CTA c of gridDim.x takes units
    // [c U / G, (c + 1) U / G) of the U = (N / 128) x (K / 128) (row tile,
    // k-step) units in row-tile order -- at most two row tiles, whose sums it
    // adds to split_acc
    int stream;
};

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major operand in the 128-byte
// swizzle layout: 8-row groups of 1024 bytes (stride byte offset 1024), the
// leading byte offset unused (encoded 16 bytes), descriptor version 1,
// layout type 2 (SWIZZLE_128B). The tile base is 1024-byte aligned.
__device__ __forceinline__ uint64_t sw128_desc(const void* tile) {
    return static_cast<uint64_t>((smem_addr(tile) >> 4) & 0x3FFF) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
           (2ull << 61);
}

// Instruction descriptor: D s32 (bits 4-5 = 2), A s8 (bits 7-9 = 1), B s8
// (bits 10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
template <int TOK>
__host__ __device__ constexpr uint32_t tc_idesc() {
    return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(TOK >> 3) << 17) |
           (static_cast<uint32_t>(kTcRows >> 4) << 24);
}

__device__ __forceinline__ void tc_mma_i8(uint32_t tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// The same with A (the unpacked weights) in tensor memory: row = lane, four
// int8 codes per 32-bit column in k order.
__device__ __forceinline__ void tc_mma_i8_ts(uint32_t tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(tmem), "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Two packed bytes of w (picked by the byte_perm selector: 0x1100 the low
// pair, 0x3322 the high pair) -> signed int8 codes lo0 hi0 lo1 hi1. With one
// 4-bit two's-complement code t per byte, t + (t & 8) * 0x1E sets the high
// nibble of exactly the negative codes (8 * 0x1E = 0xF0, no carry between
// bytes): the sign extension in one AND and one multiply-add.
__device__ __forceinline__ uint32_t nib_s8(uint32_t w, uint32_t selector) {
    const uint32_t b = __byte_perm(w, 0, selector);
    const uint32_t t = (b & 0x000F000Fu) | ((b >> 4) & 0x0F000F00u);
    return t + (t & 0x08080808u) * 0x1Eu;
}

template <int TOK>
__global__ void __launch_bounds__(TcCfg<TOK>::kThreads, 1)
    int4_gemm_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                        const TcArgs g) {
    using C = TcCfg<TOK>;
    extern __shared__ uint8_t tc_smem_raw[];
    // 1024-byte aligned base, by offsetting the shared array itself (an
    // integer round trip would hide the address space and turn every tile
    // access into a generic load or store)
    uint8_t* smem = tc_smem_raw + ((1024u - (smem_addr(tc_smem_raw) & 1023u)) & 1023u);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarrierOff);  // TMA stage landed
    uint64_t* empty = full + C::kStages;  // stage s and unpacked tile s consumed by the MMAs
    uint64_t* aready = empty + C::kStages;                                 // unpacked tile s written
    uint64_t* accfull = aready + C::kASlots;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accfull + 1);
    volatile int* failed = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // token tiles fastest: the CTAs running at once share weight tiles and
    // spread their reads of the larger activation tiles over several of them
    int n0 = blockIdx.y * kTcRows, m0 = blockIdx.x * TOK;
    // this CTA's iterations: [0, len0) are k-steps kbeg, kbeg + 1, ... of row
    // tile n0 (split-K over gridDim.z: one K slice), [len0, steps) k-steps
    // 0, 1, ... of the next row tile (stream-K only)
    const int all_steps = g.K / kTcK;
    int kbeg, steps;
    if (TOK == 64 && g.stream) {
        const long long units = static_cast<long long>(g.N / kTcRows) * all_steps;
        const long long u0 = blockIdx.x * units / gridDim.x, u1 = (blockIdx.x + 1) * units / gridDim.x;
        const int tile = static_cast<int>(u0 / all_steps);
        kbeg = static_cast<int>(u0 - static_cast<long long>(tile) * all_steps);
        steps = static_cast<int>(u1 - u0);
        n0 = tile * kTcRows;
        m0 = 0;
    } else {
        kbeg = static_cast<int>(static_cast<long long>(blockIdx.z) * all_steps / gridDim.z);
        steps = static_cast<int>(static_cast<long long>(blockIdx.z + 1) * all_steps / gridDim.z) - kbeg;
    }
    const int len0 = min(steps, all_steps - kbeg);
    const int n1 = n0 + kTcRows;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < C::kASlots; ++a) mbar_init(&aready[a], kTcGroupWarps);
        mbar_init(accfull, 1);
        *failed = wait_failed_before() ? 1 : 0;
        fence_mbar_init();
    }
    if (warp == C::kProducerWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_addr(tmem_slot)), "r"(C::kTmemCols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    auto stage = [&](int s) { return smem + s * C::kStageBytes; };

    // Every waiter below meets each barrier's phases in order (a parity wait
    // cannot tell a phase from the one two rounds later): the producer and
    // the MMA thread walk all iterations in order; unpack group g handles
    // iterations g, g + kGroups, ..., whose TMA stages (it % kStages, a
    // multiple of kGroups apart) and unpacked tiles (g, g + kGroups, used
    // in turn) are its own.
    if (warp == C::kProducerWarp) {
        if (lane == 0) {  // TMA producer
            int issued = 0;
            if (!*failed) {
                asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&wmap)) : "memory");
                asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&xmap)) : "memory");
                for (int it = 0; it < steps; ++it) {
                    const int s = it % C::kStages;
                    const uint32_t round = it / C::kStages;
                    if (*failed) break;
                    if (it >= C::kStages && !mbar_wait(&empty[s], (round - 1) & 1)) {
                        *failed = 1;
                        break;
                    }
                    const bool next = it >= len0;
                    const int kstep = next ? it - len0 : kbeg + it;
                    mbar_arrive_expect_tx(&full[s], C::kPackedBytes + C::kBBytes);
                    tma_load_2d(stage(s) + C::kPackedOff, &wmap, kstep * (kTcK / 2), next ? n1 : n0, &full[s]);
                    tma_load_2d(stage(s) + C::kBOff, &xmap, kstep * kTcK, m0, &full[s]);
                    issued = it + 1;
                }
            }
            // the copies issued must land before the CTA may exit
            for (int it = issued > C::kStages ? issued - C::kStages : 0; it < issued; ++it)
                mbar_wait(&full[it % C::kStages], (it / C::kStages) & 1);
        }
    } else if (warp == C::kMmaWarp) {
        if (lane == 0) {  // MMA issuer
            constexpr uint32_t idesc = tc_idesc<TOK>();
            for (int it = 0; it < steps && !*failed; ++it) {
                // tile s is unpacked by a group that waited for stage s to
                // land, so its aready (acquired here) covers the TMA's
                // activation tile as well
                const int s = it % C::kStages;
                if (!mbar_wait(&aready[s], (it / C::kStages) & 1)) {
                    *failed = 1;
                    break;
                }
                tc_fence_after();
                const uint64_t bdesc = sw128_desc(stage(s) + C::kBOff);
                const uint32_t atmem = tmem + C::kACol + 32 * s;
                // the second row tile of a stream-K range: the second accumulator
                const bool next = it >= len0;
                const uint32_t dtmem = tmem + (next ? TOK : 0);
                const int first = next ? len0 : 0;
#pragma unroll
                for (int kk = 0; kk < kTcK / 32; ++kk)  // K = 32: 8 columns of A, +32 bytes (+2) along B
                    tc_mma_i8_ts(dtmem, atmem + 8 * kk, bdesc + 2 * kk, idesc, (it != first) || kk != 0);
                tc_commit(&empty[s]);  // stage s and tile s free again
            }
            tc_commit(accfull);  // arrives once every MMA issued above has completed
        }
    } else {  // unpack groups, then the epilogue
        // group g = warp / 4; the warp's lane quarter (warp % 4) holds weight
        // rows 32 (warp % 4) + lane of the tile, one row per thread
        const int group = warp / kTcGroupWarps, quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
        for (int it = group; it < steps; it += C::kGroups) {
            const int s = it % C::kStages;  // the TMA stage and the unpacked tile
            const int k = it / C::kStages;  // their use count
            const bool ok = __all_sync(0xffffffffu, !*failed && (k == 0 || mbar_wait(&empty[s], (k - 1) & 1)) &&
                                                        mbar_wait(&full[s], k & 1));
            if (!ok) {
                if (lane == 0) *failed = 1;
                break;
            }
            tc_fence_after();
            // the packed tile lands 64-byte swizzled: chunk c of row r at
            // r * 64 + 16 (c ^ ((r >> 1) & 3)), so a warp's rows hit distinct banks
            const uint8_t* prow = stage(s) + C::kPackedOff + row * 64;
            uint32_t codes[32];
#pragma unroll
            for (int c = 0; c < 4; ++c) {  // 16 packed bytes = 32 codes = 8 columns
                const uint4 w = *reinterpret_cast<const uint4*>(prow + ((c ^ ((row >> 1) & 3)) << 4));
                codes[8 * c + 0] = nib_s8(w.x, 0x1100);
                codes[8 * c + 1] = nib_s8(w.x, 0x3322);
                codes[8 * c + 2] = nib_s8(w.y, 0x1100);
                codes[8 * c + 3] = nib_s8(w.y, 0x3322);
                codes[8 * c + 4] = nib_s8(w.z, 0x1100);
                codes[8 * c + 5] = nib_s8(w.z, 0x3322);
                codes[8 * c + 6] = nib_s8(w.w, 0x1100);
                codes[8 * c + 7] = nib_s8(w.w, 0x3322);
            }
            const uint32_t acol = lane_base + C::kACol + 32 * s;
#pragma unroll
            for (int h = 0; h < 2; ++h)
                asm volatile(
                    "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
                    "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
                    ::"r"(acol + 16 * h), "r"(codes[16 * h + 0]), "r"(codes[16 * h + 1]), "r"(codes[16 * h + 2]),
                      "r"(codes[16 * h + 3]), "r"(codes[16 * h + 4]), "r"(codes[16 * h + 5]), "r"(codes[16 * h + 6]),
                      "r"(codes[16 * h + 7]), "r"(codes[16 * h + 8]), "r"(codes[16 * h + 9]), "r"(codes[16 * h + 10]),
                      "r"(codes[16 * h + 11]), "r"(codes[16 * h + 12]), "r"(codes[16 * h + 13]),
                      "r"(codes[16 * h + 14]), "r"(codes[16 * h + 15])
                    : "memory");
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();  // tensor-memory stores -> ordered before the MMAs that read them
            __syncwarp();
            if (lane == 0) mbar_arrive(&aready[s]);
        }
        // epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 = weight rows n0 + 32 (w % 4) + lane,
        // columns (tokens) of slice w / 4
        const bool done = __all_sync(0xffffffffu, mbar_wait(accfull, 0) && !*failed);
        tc_fence_after();
        if (done && warp < 16 && steps > 0) {  // the first sixteen warps: four column slices per lane quarter
            constexpr int kSlices = 4, kCols = TOK / kSlices;
            static_assert(kCols % 16 == 0, "column slices of whole 16-column loads");
            const int quarter = warp & 3, slice = warp >> 2;
            if (TOK == 64 && g.stream) {
                // stream-K: each row tile's sums (1 or 2 accumulators) into split_acc
                for (int t = 0; t < (steps > len0 ? 2 : 1); ++t) {
                    const int row = (t ? n1 : n0) + quarter * 32 + lane;
                    const uint32_t base = tmem + t * TOK + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll 1
                    for (int c0 = slice * kCols; c0 < (slice + 1) * kCols; c0 += 16) {
                        uint32_t v[16];
                        tmem_ld16(base + c0, v);
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            if (c0 + j < g.M)
                                atomicAdd(g.split_acc + static_cast<size_t>(c0 + j) * g.N + row, static_cast<int>(v[j]));
                    }
                }
            } else {
            const int row = n0 + quarter * 32 + lane;
            const float ws = g.w_scale[row];
            const uint32_t base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll 1
            for (int c0 = slice * kCols; c0 < (slice + 1) * kCols; c0 += 16) {
                uint32_t v[16];
                tmem_ld16(base + c0, v);
                if (g.split_acc || g.out_i32) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int m = m0 + c0 + j;
                        if (m >= g.M) continue;
                        if (g.split_acc)
                            atomicAdd(g.split_acc + static_cast<size_t>(m) * g.N + row, static_cast<int>(v[j]));
                        else
                            g.out_i32[static_cast<size_t>(m) * g.N + row] = static_cast<int>(v[j]);
                    }
                    continue;
                }
                // every load (token scales, residual values) before the first
                // store, so the loads overlap instead of queueing behind the
                // stores they might alias
                const float as_lane = g.act_scale[min(m0 + c0 + (lane & 15), g.M - 1)];
                float prev[16];
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    prev[j] = g.residual ? g.out[static_cast<size_t>(min(m0 + c0 + j, g.M - 1)) * g.N + row] : 0.f;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int m = m0 + c0 + j;
                    const float as = __shfl_sync(0xffffffffu, as_lane, j);
                    if (m >= g.M) continue;
                    const float value = __fmul_rn(__fmul_rn(static_cast<float>(static_cast<int>(v[j])), as), ws);
                    g.out[static_cast<size_t>(m) * g.N + row] = g.residual ? __fadd_rn(prev[j], value) : value;
                }
            }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == C::kProducerWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::kTmemCols)
                     : "memory");
    }
}

}  // namespace h4b

#include <mutex>
#include <unordered_map>

namespace h4b {

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against libcuda); encoded maps are cached per (address, shape, box).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }();
    return fn;
}

struct MapKey {
    const void* base;
    uint64_t inner, outer;
    uint32_t box_inner, box_outer, swizzle;
    bool operator==(const MapKey& o) const {
        return base == o.base && inner == o.inner && outer == o.outer && box_inner == o.box_inner &&
               box_outer == o.box_outer && swizzle == o.swizzle;
    }
};
struct MapKeyHash {
    size_t operator()(const MapKey& k) const {
        size_t h = reinterpret_cast<uintptr_t>(k.base);
        for (uint64_t v : {k.inner, k.outer, uint64_t(k.box_inner) << 32 | k.box_outer, uint64_t(k.swizzle)})
            h = h * 1000003u ^ static_cast<size_t>(v);
        return h;
    }
};

// A row-major uint8 matrix [outer][inner] as a 2-D tensor map with box
// [box_outer][box_inner]; rows past `outer` read as zeros.
bool byte_matrix_map(CUtensorMap* out, const void* base, uint64_t inner, uint64_t outer, uint32_t box_inner,
                     uint32_t box_outer, int swizzle_bytes) {
    static std::mutex lock;
    static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
    const MapKey key{base, inner, outer, box_inner, box_outer, static_cast<uint32_t>(swizzle_bytes)};
    std::lock_guard<std::mutex> guard(lock);
    auto hit = cache.find(key);
    if (hit != cache.end()) {
        *out = hit->second;
        return true;
    }
    auto encode = tensor_map_encoder();
    if (!encode) return false;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {inner};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t elem[2] = {1, 1};
    if (encode(out, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, elem,
               CU_TENSOR_MAP_INTERLEAVE_NONE,
               swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                    : (swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE),
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    if (cache.size() > 8192) cache.clear();
    cache.emplace(key, *out);
    return true;
}

// out[m][n] = float(acc) * act_scale[m] * w_scale[n] (the GEMM epilogue's
// order; with `residual`, added to out[m][n]) from the split-K sums, which it
// leaves zero for the next GEMM.
__global__ void split_finalize_kernel(int32_t* acc, const float* act_scale, const float* w_scale, float* out, int M,
                                      int N, int residual) {
    const long long total = static_cast<long long>(M) * N;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int m = static_cast<int>(i / N), n = static_cast<int>(i - static_cast<long long>(m) * N);
        const float value = __fmul_rn(__fmul_rn(static_cast<float>(acc[i]), act_scale[m]), w_scale[n]);
        out[i] = residual ? __fadd_rn(out[i], value) : value;
        acc[i] = 0;
    }
}

// The same, four columns per thread, row m = blockIdx.y (N % 4 == 0 and
// acc, w_scale, out 16-byte aligned).
__global__ void split_finalize_vec_kernel(int32_t* acc, const float* act_scale, const float* w_scale, float* out,
                                          int N, int residual) {
    const int m = blockIdx.y;
    const int n = 4 * (blockIdx.x * blockDim.x + threadIdx.x);
    if (n >= N) return;
    const size_t i = static_cast<size_t>(m) * N + n;
    const int4 sum = *reinterpret_cast<const int4*>(acc + i);
    const float4 ws = *reinterpret_cast<const float4*>(w_scale + n);
    const float as = act_scale[m];
    const float4 prev = residual ? *reinterpret_cast<const float4*>(out + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    auto value = [&](int v, float w, float p) {
        const float x = __fmul_rn(__fmul_rn(static_cast<float>(v), as), w);
        return residual ? __fadd_rn(p, x) : x;
    };
    *reinterpret_cast<float4*>(out + i) =
        make_float4(value(sum.x, ws.x, prev.x), value(sum.y, ws.y, prev.y), value(sum.z, ws.z, prev.z),
                    value(sum.w, ws.w, prev.w));
    *reinterpret_cast<int4*>(acc + i) = make_int4(0, 0, 0, 0);
}

bool tc_gemm_supported(const GemmArgs& g) {
    return g.N % kTcRows == 0 && g.K % kTcK == 0 && (reinterpret_cast<uintptr_t>(g.w) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(g.x) & 15) == 0 && tensor_map_encoder() != nullptr;
}

template <int TOK>
int launch_tc(const GemmArgs& g, cudaStream_t stream) {
    using C = TcCfg<TOK>;
    // The shared-memory opt-in applies to the current device only: set it
    // once per device, recording only a success.
    static std::atomic<bool> opted_in[kMaxDevices];
    int dev = 0;
    H4B_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return H4B_EUNSUPPORTED;
    if (!opted_in[dev].load(std::memory_order_acquire)) {
        H4B_CUDA_TRY(cudaFuncSetAttribute(int4_gemm_tc_kernel<TOK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          C::kSmem));
        opted_in[dev].store(true, std::memory_order_release);
    }
    CUtensorMap wmap, xmap;
    if (!byte_matrix_map(&wmap, g.w, static_cast<uint64_t>(g.K) / 2, g.N, kTcK / 2, kTcRows, 64) ||
        !byte_matrix_map(&xmap, g.x, g.K, g.M, kTcK, TOK, 128))
        return H4B_EUNSUPPORTED;
    // With the caller's zeroed int32 buffer (split_acc) the int32 sums are
    // added there (exact in any order) and finalised below:
    // * M <= 64: stream-K, one CTA per SM over the (row tile, k-step) units,
    //   when that gives every CTA at most K / 128 + 1 units (two row tiles):
    //   all SMs busy for the same number of k-steps whatever the tile count
    //   (gate_up's 152 row tiles are two waves of one CTA per SM otherwise);
    // * else few output tiles (under half the SMs): split K so the grid fills
    //   the SMs, each slice at least 4 k-steps.
    const int tiles = (g.N / kTcRows) * ((g.M + TOK - 1) / TOK);
    const int steps = g.K / kTcK;
    int ksplit = 1, stream_ctas = 0;
    if (g.split_acc && !g.out_i32) {
        const long long units = static_cast<long long>(tiles) * steps;
        const long long ctas = std::min<long long>(sm_count(), units);
        if (TOK == 64 && g.M <= TOK && (units + ctas - 1) / ctas <= steps + 1)
            stream_ctas = static_cast<int>(ctas);
        else if (tiles < sm_count() / 2)
            ksplit = std::max(1, std::min(sm_count() / tiles, steps / 4));
    }
    const bool accumulate = stream_ctas > 0 || ksplit > 1;
    const TcArgs a{g.act_scale, g.w_scale, g.out, g.M, g.N, g.K, g.out_i32, accumulate ? g.split_acc : nullptr,
                   g.residual ? 1 : 0, stream_ctas > 0 ? 1 : 0};
    const dim3 grid = stream_ctas > 0 ? dim3(stream_ctas, 1, 1) : dim3((g.M + TOK - 1) / TOK, g.N / kTcRows, ksplit);
    int4_gemm_tc_kernel<TOK><<<grid, C::kThreads, C::kSmem, stream>>>(wmap, xmap, a);
    H4B_CUDA_TRY(cudaGetLastError());
    if (g.finalize_deferred) *g.finalize_deferred = accumulate;
    if (accumulate && !g.finalize_deferred) {
        const long long n = static_cast<long long>(g.M) * g.N;
        const bool aligned = ((reinterpret_cast<uintptr_t>(g.split_acc) | reinterpret_cast<uintptr_t>(g.w_scale) |
                               reinterpret_cast<uintptr_t>(g.out)) & 15) == 0;
        if (aligned && g.N % 4 == 0 && g.M <= 65535)
            split_finalize_vec_kernel<<<dim3((g.N / 4 + 255) / 256, g.M), 256, 0, stream>>>(
                g.split_acc, g.act_scale, g.w_scale, g.out, g.N, g.residual ? 1 : 0);
        else
            split_finalize_kernel<<<static_cast<int>(std::min<long long>((n + 255) / 256, 8ll * sm_count())), 256, 0,
                                    stream>>>(g.split_acc, g.act_scale, g.w_scale, g.out, g.M, g.N,
                                             g.residual ? 1 : 0);
        H4B_CUDA_TRY(cudaGetLastError());
    }
    return 0;
}

// kernel: 0 = tensor-core tcgen05 where the shape allows it (N % 128, K % 128),
// else mma.sync; 1 = tcgen05 only; 2 = mma.sync only.
int launch_int4_gemm(const GemmArgs& g, cudaStream_t stream, int kernel = 0) {
    if (g.M < 1 || g.N < 1 || g.K < 1) return H4B_EINVAL;
    if (kernel < 0 || kernel > 2) return H4B_EINVAL;
    if (g.finalize_deferred) *g.finalize_deferred = false;  // the mma.sync kernel writes out directly
    if (kernel == 2 || (kernel == 0 && !tc_gemm_supported(g))) return launch_int4_gemm_mma(g, stream);
    if (!tc_gemm_supported(g)) return H4B_EUNSUPPORTED;
    if (g.M <= 64) return launch_tc<64>(g, stream);
    if (g.M <= 128) return launch_tc<128>(g, stream);
    return launch_tc<256>(g, stream);
}

}  // namespace h4b

extern "C" int h4b_quantize_rows(const float* values, int8_t* quantized, float* scales, int32_t* sums, int rows,
                                 int width, void* stream) {
    if (!values || !quantized || !scales || !sums || rows < 1 || width < 1) return H4B_EINVAL;
    h4b::quantize_rows_kernel<<<rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(values, width, quantized, scales,
                                                                                 sums);
    H4B_CUDA_TRY(cudaGetLastError());
    return 0;
}

extern "C" int h4b_int4_gemm_ex(const int8_t* x8, const float* act_scales, const int32_t* act_sums,
                                const uint8_t* weights, const float* scales, float* output, int tokens, int rows,
                                int width, int kernel, void* stream) {
    if (!x8 || !act_scales || !act_sums || !weights || !scales || !output) return H4B_EINVAL;
    h4b::GemmArgs g{x8, act_scales, act_sums, weights, scales, output, tokens, rows, width};
    return h4b::launch_int4_gemm(g, static_cast<cudaStream_t>(stream), kernel);
}

extern "C" int h4b_int4_gemm(const int8_t* x8, const float* act_scales, const int32_t* act_sums, const uint8_t* weights,
                             const float* scales, float* output, int tokens, int rows, int width, void* stream) {
    return h4b_int4_gemm_ex(x8, act_scales, act_sums, weights, scales, output, tokens, rows, width, 0, stream);
}

extern "C" int h4b_int4_gemm_acc(const int8_t* x8, const float* act_scales, const int32_t* act_sums,
                                 const uint8_t* weights, const float* scales, float* output, int32_t* acc, int tokens,
                                 int rows, int width, int residual, void* stream) {
    if (!x8 || !act_scales || !act_sums || !weights || !scales || !output || !acc) return H4B_EINVAL;
    if ((reinterpret_cast<uintptr_t>(acc) & 3) != 0) return H4B_EINVAL;
    h4b::GemmArgs g{x8, act_scales, act_sums, weights, scales, output, tokens, rows, width};
    g.split_acc = acc;
    g.residual = residual != 0;
    return h4b::launch_int4_gemm(g, static_cast<cudaStream_t>(stream), 0);
}
