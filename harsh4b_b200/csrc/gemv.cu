// Packed signed-int4 x int8 GEMV for batch-1 decode on sm_100a.
//
// Computes, for each weight row r (reference: cpu_kernels/litespark_int4.cpp:22-76),
//   acc[r] = sum_k w4[r,k] * x8[k]                       (exact int32)
//   out[r] = float(acc[r]) * act_scale * w_scale[r]       (left to right)
// with the int8 activation produced inside the kernel (fused prologue) and
// the consumer of out fused into the epilogue.
//
// Data movement: one CTA per SM owns a contiguous range of rows. Its rows
// are one contiguous byte range of the row-major weight matrix, so a
// producer warp streams them with 1-D bulk copies (the TMA engine) into a
// ring of shared-memory stages tracked by mbarriers. The first ring's worth
// is issued before griddepcontrol.wait: weights do not depend on the
// previous kernel, so under programmatic dependent launch each GEMV's weight
// stream overlaps the previous kernel's tail.
//
// Work split: the consumer warps own ring tiles round-robin (tile t belongs
// to warp t % 8) and process a tile's rows in batches with independent
// accumulators, so the fixed per-tile latencies (barrier wait, the row
// reductions) are paid once per batch, not once per row.
//
// Math: a lane owns a fixed set of 16-byte weight chunks (32 codes) of
// every row, so up to K = 4096 its 32-byte activation slices live in
// registers for the whole kernel (above that they are re-read from shared
// memory). Each 4-byte weight word holds 8 codes;
// reading a nibble n as u = n ^ 8 = s + 8 (0..15) turns the even and odd
// codes into two dp4a operands with no sign extension, and the bias
// 8 * sum(x) is folded into the lane's starting accumulator.
#include <cstdlib>

#include "common.cuh"

namespace h4b {

enum { PRO_INT8 = 0, PRO_QUANT = 1, PRO_QUANT_ABSMAX = 2, PRO_RMSNORM = 3 };
enum { EPI_STORE = 0, EPI_RESIDUAL = 1, EPI_SWIGLU = 2, EPI_ARGMAX = 3 };

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kGemvThreads = kConsumers + 32;
constexpr int kMaxStages = 16;
constexpr int kMaxSlots = 16;       // K <= 16384
constexpr int kMaxRegSlots = 4;     // activation in registers up to K = 4096
constexpr int kSwigluBlock = 4;  // gate/up interleave block (rows)
constexpr int kRingBytes = 96 * 1024;
constexpr int kStageTarget = 16 * 1024;

struct GemvArgs {
    const uint8_t* w;
    const float* wscale;
    int rows, width;
    int row_align;      // rows per partition unit (2 * kSwigluBlock for SwiGLU)
    int tile_rows;      // rows per ring stage
    int stages;         // ring depth
    int rows_cap;       // smem rows reserved per CTA (multiple of 32)
    const int8_t* x8;   // PRO_INT8 input
    const float* xin;   // fp32 input
    const float* gamma; // PRO_RMSNORM weight
    const float* absmax_in;  // PRO_QUANT_ABSMAX
    float act_scale;    // PRO_INT8
    float eps;
    float* out;
    int32_t* acc_out;
    float* act_scale_out;
    float* absmax_out;
    unsigned long long* argmax_out;
};

// Bytes reserved for the quantised activation: rounded up to whole slots
// (32 lanes x 32 B) plus 3 slots, the most an instantiated slot count
// exceeds the needed one.
__host__ __device__ inline int xq_region(int width) { return ((width + 1023) & ~1023) + 3072; }

struct SmemLayout {
    int red, xq, gamma, acc, scale, ring, total;
};

__host__ __device__ inline SmemLayout smem_layout(int width, int rows_cap, int stages, int stage_bytes,
                                                  bool with_gamma) {
    SmemLayout s;
    s.red = 2 * kMaxStages * 8;               // barriers first
    s.xq = s.red + 64 * 4;                    // 32 floats + flags
    s.gamma = s.xq + xq_region(width);
    s.acc = s.gamma + (with_gamma ? width * 4 : 0);
    s.scale = s.acc + rows_cap * 4;
    s.ring = (s.scale + rows_cap * 4 + 127) & ~127;
    s.total = s.ring + stages * stage_bytes + 512;  // slot loads may run up to 496 B past a tile
    return s;
}

__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// One 16-byte weight chunk (32 codes) against the lane's 32 activation
// bytes. Word j pairs with the activation words (even, odd) of column group
// j. A nibble n is read as u = n ^ 8 = s + 8: the low nibbles of a word
// masked in place are 4 unsigned bytes u, the high nibbles masked in place
// are 4 unsigned bytes 16u, so each word costs two LOP3 and two u8 x s8
// dp4a, and the high sum is an exact multiple of 16 (see row_total).
__device__ __forceinline__ void dot_chunk(const uint4 w, const uint4 xa, const uint4 xb, int lo[4], int hi[4]) {
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
    const uint32_t xe[4] = {xa.x, xa.z, xb.x, xb.z};
    const uint32_t xo[4] = {xa.y, xa.w, xb.y, xb.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t u = ww[j] ^ 0x88888888u;
        lo[j] = dp4a_us(u & 0x0F0F0F0Fu, xe[j], lo[j]);
        hi[j] = dp4a_us(u & 0xF0F0F0F0u, xo[j], hi[j]);
    }
}

// A lane's share of one row: sum u*x over its codes minus 8 * sum(x) (bias).
__device__ __forceinline__ int row_total(const int lo[4], const int hi[4], int bias) {
    return bias + ((lo[0] + lo[1]) + (lo[2] + lo[3])) + (((hi[0] + hi[1]) + (hi[2] + hi[3])) >> 4);
}

// Row sums for rows b0 .. b0+RB-1 of a tile (a short batch repeats its last
// row). Loads are unconditional: lanes past the row end read padding or the
// next row and multiply it by zero activations.
template <int SLOTS, int RB, bool XREG>
__device__ __forceinline__ void tile_batch(const uint8_t* tile, int kb, int trows, int b0, const uint4* xa,
                                           const uint4* xb, const int8_t* xq, int lane, int bias, int total[RB]) {
    int lo[RB][4], hi[RB][4];
#pragma unroll
    for (int i = 0; i < RB; ++i)
#pragma unroll
        for (int q = 0; q < 4; ++q) lo[i][q] = hi[i][q] = 0;
#pragma unroll
    for (int j = 0; j < SLOTS; ++j) {
        const int c = lane + 32 * j;
        uint4 va, vb;
        if constexpr (XREG) {
            va = xa[j];
            vb = xb[j];
        } else {
            va = *reinterpret_cast<const uint4*>(xq + 32 * c);
            vb = *reinterpret_cast<const uint4*>(xq + 32 * c + 16);
        }
#pragma unroll
        for (int i = 0; i < RB; ++i) {
            const int lr = min(b0 + i, trows - 1);
            const uint4 w = *reinterpret_cast<const uint4*>(tile + static_cast<size_t>(lr) * kb + 16 * c);
            dot_chunk(w, va, vb, lo[i], hi[i]);
        }
    }
#pragma unroll
    for (int i = 0; i < RB; ++i) total[i] = __reduce_add_sync(0xffffffffu, row_total(lo[i], hi[i], bias));
}

// Zero xq past the activation to the end of its region, so the unconditional
// slot loads of the shared-memory activation path read zeros.
__device__ __forceinline__ void zero_xq_tail(int8_t* xq, int n, int tid, int nthreads) {
    const int end = xq_region(n);
    #pragma unroll 1
    for (int i = n + 4 * tid; i < end; i += 4 * nthreads) *reinterpret_cast<uint32_t*>(xq + i) = 0u;
}

// Writes the 8 quantised values of group g (columns 8g..8g+7) as
// [x0 x2 x4 x6][x1 x3 x5 x7] at xq + 8g.
__device__ __forceinline__ void store_group(int8_t* xq, int g, const int q[8]) {
    const uint32_t even = (q[0] & 0xFF) | ((q[2] & 0xFF) << 8) | ((q[4] & 0xFF) << 16) | ((uint32_t)(q[6] & 0xFF) << 24);
    const uint32_t odd = (q[1] & 0xFF) | ((q[3] & 0xFF) << 8) | ((q[5] & 0xFF) << 16) | ((uint32_t)(q[7] & 0xFF) << 24);
    *reinterpret_cast<uint2*>(xq + 8 * g) = make_uint2(even, odd);
}

__device__ __forceinline__ void load8(const float* p, float v[8]) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// Builds the permuted int8 activation in shared memory; returns the dequant
// scale. Runs on the consumer warps only (named barrier 1).
template <int PRO>
__device__ float gemv_prologue(const GemvArgs& a, int8_t* xq, float* red, const float* gamma_s) {
    const int tid = threadIdx.x;
    const int groups = a.width >> 3;
    if constexpr (PRO == PRO_INT8) {
        #pragma unroll 2
        for (int g = tid; g < groups; g += kConsumers) {
            const uint2 raw = *reinterpret_cast<const uint2*>(a.x8 + 8 * g);
            int q[8];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                q[e] = static_cast<int8_t>((raw.x >> (8 * e)) & 0xFF);
                q[4 + e] = static_cast<int8_t>((raw.y >> (8 * e)) & 0xFF);
            }
            store_group(xq, g, q);
        }
        zero_xq_tail(xq, a.width, tid, kConsumers);
        return a.act_scale;
    } else {
        float inv = 1.0f;
        if constexpr (PRO == PRO_RMSNORM) {
            float ss = 0.f;
            #pragma unroll 2
            for (int g = tid; g < groups; g += kConsumers) {
                float v[8];
                load8(a.xin + 8 * g, v);
#pragma unroll
                for (int e = 0; e < 8; ++e) ss = __fmaf_rn(v[e], v[e], ss);
            }
            ss = group_sum(ss, red, kConsumerWarps, 1);
            const float mean = __fdiv_rn(ss, static_cast<float>(a.width));
            inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
        }
        float m;
        if constexpr (PRO == PRO_QUANT_ABSMAX) {
            m = *a.absmax_in;
        } else {
            float local = 0.f;
            #pragma unroll 2
            for (int g = tid; g < groups; g += kConsumers) {
                float v[8], gm[8];
                load8(a.xin + 8 * g, v);
                if constexpr (PRO == PRO_RMSNORM) load8(gamma_s + 8 * g, gm);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float n = (PRO == PRO_RMSNORM) ? __fmul_rn(__fmul_rn(v[e], inv), gm[e]) : v[e];
                    local = fmaxf(local, fabsf(n));
                }
            }
            m = group_max(local, red, kConsumerWarps, 1);
        }
        const float qs = quant_multiplier(m);
#pragma unroll 2
        for (int g = tid; g < groups; g += kConsumers) {
            float v[8], gm[8];
            int q[8];
            load8(a.xin + 8 * g, v);
            if constexpr (PRO == PRO_RMSNORM) load8(gamma_s + 8 * g, gm);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float n = (PRO == PRO_RMSNORM) ? __fmul_rn(__fmul_rn(v[e], inv), gm[e]) : v[e];
                q[e] = quantize_one(n, qs);
            }
            store_group(xq, g, q);
        }
        zero_xq_tail(xq, a.width, tid, kConsumers);
        return dequant_scale(m);
    }
}

template <int PRO, int EPI, int SLOTS>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int kb = a.width >> 1;
    const uint32_t stage_bytes = static_cast<uint32_t>(a.tile_rows) * kb;
    const SmemLayout L = smem_layout(a.width, a.rows_cap, a.stages, stage_bytes, PRO == PRO_RMSNORM);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kMaxStages;
    float* red = reinterpret_cast<float*>(smem + L.red);
    int* flags = reinterpret_cast<int*>(red + 32);  // [0] error, [1] act scale bits, [2] skip
    int8_t* xq = reinterpret_cast<int8_t*>(smem + L.xq);
    int32_t* acc_s = reinterpret_cast<int32_t*>(smem + L.acc);
    float* sc_s = reinterpret_cast<float*>(smem + L.scale);
    uint8_t* ring = smem + L.ring;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int units = a.rows / a.row_align;
    const int u0 = static_cast<int>(static_cast<long long>(blockIdx.x) * units / gridDim.x);
    const int u1 = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * units / gridDim.x);
    const int r0 = u0 * a.row_align;
    const int nrows = (u1 - u0) * a.row_align;
    const int ntiles = (nrows + a.tile_rows - 1) / a.tile_rows;

    if (tid == 0) {
        for (int s = 0; s < a.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);  // released by the tile's owning warp
        }
        flags[0] = 0;
        flags[2] = wait_failed_before();
        fence_mbar_init();
    }
    __syncthreads();
    pdl_trigger();
    if (flags[2]) return;  // before any bulk copy is issued

    if (warp == kConsumerWarps) {
        // ---------------- producer warp ----------------
        int issued = 0;
        auto issue = [&](int t) {
            const int s = t % a.stages;
            const int rows_t = min(a.tile_rows, nrows - t * a.tile_rows);
            const uint32_t bytes = static_cast<uint32_t>(rows_t) * kb;
            mbar_arrive_expect_tx(&full[s], bytes);
            bulk_g2s(ring + static_cast<size_t>(s) * stage_bytes,
                     a.w + static_cast<size_t>(r0 + t * a.tile_rows) * kb, bytes, &full[s]);
        };
        if (lane == 0) {
            const int first = min(a.stages, ntiles);
            for (int t = 0; t < first; ++t) issue(t);
            issued = first;
        }
        // Row scales are weights too: fetch them asynchronously before any
        // dependency wait, so lane 0 goes straight on to refilling the ring.
        #pragma unroll 1
        for (int i = lane; i < nrows; i += 32) async_copy4(sc_s + i, a.wscale + r0 + i);
        if (lane == 0) {
            for (int t = a.stages; t < ntiles; ++t) {
                const int s = t % a.stages;
                if (!mbar_wait(&empty[s], ((t / a.stages) - 1) & 1)) {
                    atomicOr(&flags[0], 1);
                    break;
                }
                issue(t);
                issued = t + 1;
            }
            // Never leave the CTA with bulk copies in flight.
            for (int t = max(0, issued - a.stages); t < issued; ++t)
                mbar_wait(&full[t % a.stages], (t / a.stages) & 1, 100000000ull);
        }
        async_copy_wait_all();
    } else {
        // ---------------- consumer warps ----------------
        float* gamma_s = reinterpret_cast<float*>(smem + L.gamma);
        if constexpr (PRO == PRO_RMSNORM) {
            // The norm weight is static: stage it before the dependency wait.
            #pragma unroll 1
            for (int i = tid; i < (a.width >> 2); i += kConsumers)
                reinterpret_cast<float4*>(gamma_s)[i] = __ldg(reinterpret_cast<const float4*>(a.gamma) + i);
        }
        pdl_wait();
        const float act_scale = gemv_prologue<(PRO)>(a, xq, red, gamma_s);
        if (tid == 0) flags[1] = __float_as_int(act_scale);
        named_sync(1, kConsumers);

        const int chunks = a.width >> 5;
        constexpr bool kXReg = SLOTS <= kMaxRegSlots;
        constexpr int kXSlots = kXReg ? SLOTS : 1;
        constexpr int RB = 2;  // rows per batch
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

        for (int t = warp; t < ntiles; t += kConsumerWarps) {
            const int s = t % a.stages;
            if (!mbar_wait(&full[s], (t / a.stages) & 1)) {
                atomicOr(&flags[0], 1);
                break;
            }
            const uint8_t* tile = ring + static_cast<size_t>(s) * stage_bytes;
            const int trows = min(a.tile_rows, nrows - t * a.tile_rows);
            for (int b0 = 0; b0 < trows; b0 += RB) {
                int total[RB];
                tile_batch<SLOTS, RB, kXReg>(tile, kb, trows, b0, xa, xb, xq, lane, bias, total);
                if (lane == 0) {
#pragma unroll
                    for (int i = 0; i < RB; ++i)
                        if (b0 + i < trows) acc_s[t * a.tile_rows + b0 + i] = total[i];
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
    }
    __syncthreads();
    if (flags[0]) return;

    // ---------------- epilogue (all threads) ----------------
    const float act_scale = __int_as_float(flags[1]);
    auto value = [&](int i) {
        return __fmul_rn(__fmul_rn(static_cast<float>(acc_s[i]), act_scale), sc_s[i]);
    };
    if constexpr (EPI == EPI_STORE || EPI == EPI_RESIDUAL) {
        #pragma unroll 1
        for (int i = tid; i < nrows; i += kGemvThreads) {
            const float v = value(i);
            if constexpr (EPI == EPI_STORE) {
                if (a.out) a.out[r0 + i] = v;
            }
            else a.out[r0 + i] = __fadd_rn(a.out[r0 + i], v);
            if (a.acc_out) a.acc_out[r0 + i] = acc_s[i];
        }
        if (a.act_scale_out && blockIdx.x == 0 && tid == 0) *a.act_scale_out = act_scale;
    } else if constexpr (EPI == EPI_SWIGLU) {
        float local = 0.f;
        const int pairs = nrows >> 1;
        #pragma unroll 1
        for (int p = tid; p < pairs; p += kGemvThreads) {
            const int b = p / kSwigluBlock, j = p % kSwigluBlock;
            const int gi = 2 * kSwigluBlock * b + j;
            const float g = value(gi), u = value(gi + kSwigluBlock);
            // cpu_lightspark.py:451-455: gate / (1 + exp(-gate)) * up
            const float act = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, exp_cw(-g))), u);
            a.out[(r0 >> 1) + p] = act;
            local = fmaxf(local, fabsf(act));
        }
        local = warp_max(local);
        if (lane == 0) red[warp] = local;
        __syncthreads();
        if (tid == 0) {
            float m = red[0];
            for (int w = 1; w < kGemvThreads / 32; ++w) m = fmaxf(m, red[w]);
            atomic_max_nonneg(a.absmax_out, m);
        }
    } else {  // EPI_ARGMAX
        unsigned long long best = 0ull;
        #pragma unroll 1
        for (int i = tid; i < nrows; i += kGemvThreads) {
            const float v = value(i);
            a.out[r0 + i] = v;
            const unsigned long long k = argmax_key(v, static_cast<uint32_t>(r0 + i));
            best = k > best ? k : best;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
            best = other > best ? other : best;
        }
        unsigned long long* keys = reinterpret_cast<unsigned long long*>(acc_s);
        __syncthreads();  // acc_s is free now
        if (lane == 0) keys[warp] = best;
        __syncthreads();
        if (tid == 0) {
            for (int w = 1; w < kGemvThreads / 32; ++w) best = keys[w] > best ? keys[w] : best;
            best = keys[0] > best ? keys[0] : best;
            atomicMax(a.argmax_out, best);
        }
    }
}

// ---------------------------------------------------------------------------
// Host-side planning and launch.

struct GemvPlan {
    int grid, slots, tile_rows, stages, rows_cap, smem;
};

// Per-device state: the SM count and whether this device's kernels have
// their shared-memory opt-ins. cudaFuncSetAttribute applies to the current
// device only, so a process that drives several GPUs prepares each one.
// Only successes are recorded; a failed preparation is retried next call.
struct DeviceSetup {
    std::atomic<int> sms{0};
    std::atomic<bool> prepared{false};
};
static DeviceSetup g_devices[kMaxDevices];
static std::mutex g_prepare_mutex;

static int current_device() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
    return dev;
}

int sm_count() {
    const int dev = current_device();
    if (dev < 0) return 148;
    int n = g_devices[dev].sms.load(std::memory_order_relaxed);
    if (n == 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        g_devices[dev].sms.store(n, std::memory_order_relaxed);
    }
    return n;
}

// Slot counts that have kernel instantiations (a lane covers `slots` 16-byte
// chunks of every row).
static int instantiated_slots(int needed) {
    static const int kSlots[] = {1, 2, 3, 4, 6, 8, 10, 12, 16};
    for (int v : kSlots)
        if (v >= needed) return v;
    return 0;
}

// Bytes of the shared-memory weight ring (tuning builds may override it
// with H4B_GEMV_RING_KB).
static int gemv_ring_bytes() {
#ifdef H4B_TUNING
    const char* e = std::getenv("H4B_GEMV_RING_KB");
    if (e && *e) return std::max(16, std::atoi(e)) * 1024;
#endif
    return kRingBytes;
}

int plan_gemv(int rows, int width, int row_align, GemvPlan* p) {
    const int ring_bytes = gemv_ring_bytes();
    if (rows <= 0 || width <= 0 || (width & 31) || rows % row_align) return H4B_EINVAL;
    const int chunks = width >> 5;
    const int slots = instantiated_slots((chunks + 31) / 32);
    if (slots == 0) return H4B_EUNSUPPORTED;
    const int kb = width >> 1;
    const int units = rows / row_align;
    const int grid = max(1, min(sm_count(), units));
    const int per_cta = ((units + grid - 1) / grid) * row_align;
    // Enough tiles per CTA for every consumer warp, at most 8 rows / 16 KB each.
    int tile_rows = max(1, min(8, (per_cta + kConsumerWarps - 1) / kConsumerWarps));
    tile_rows = max(1, min(tile_rows, kStageTarget / kb));
    // The ring depth is a multiple of the consumer warps: tile t sits in slot
    // t % stages and belongs to warp t % 8, so every slot has one owner that
    // waits on the slot's phases in order. (With a shared slot a warp could
    // start waiting for a tile while the slot's previous tile, owned by
    // another warp, is still in flight -- and the mbarrier parity of that
    // older phase would read as complete.)
    tile_rows = max(1, min(tile_rows, ring_bytes / (kConsumerWarps * kb)));
    const int stage_bytes = tile_rows * kb;
    if (stage_bytes > 64 * 1024 || kConsumerWarps * stage_bytes > ring_bytes) return H4B_EUNSUPPORTED;
    const int stages = min(kMaxStages, ring_bytes / stage_bytes) / kConsumerWarps * kConsumerWarps;
    const int rows_cap = (per_cta + 31) & ~31;
    const SmemLayout L = smem_layout(width, rows_cap, stages, stage_bytes, true);
    if (L.total > 227 * 1024) return H4B_EUNSUPPORTED;
    *p = GemvPlan{grid, slots, tile_rows, stages, rows_cap, L.total};
    return 0;
}

// Every kernel of the decode chain asks for the same (maximal) shared-memory
// carveout, so a kernel's CTAs can become resident next to its predecessor's
// under programmatic dependent launch instead of waiting for an SM to drain.
template <typename K>
int set_carveout(K kernel) {
    H4B_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                      cudaSharedmemCarveoutMaxShared));
    return 0;
}

template <int PRO, int EPI, int SLOTS>
static int set_smem_limit() {
    H4B_CUDA_TRY(cudaFuncSetAttribute(gemv_kernel<PRO, EPI, SLOTS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      227 * 1024));
    return set_carveout(gemv_kernel<PRO, EPI, SLOTS>);
}

template <int PRO, int EPI>
static int set_smem_limits() {
    int r = 0;
    if ((r = set_smem_limit<PRO, EPI, 1>()) || (r = set_smem_limit<PRO, EPI, 2>()) ||
        (r = set_smem_limit<PRO, EPI, 3>()) || (r = set_smem_limit<PRO, EPI, 4>()) ||
        (r = set_smem_limit<PRO, EPI, 6>()) || (r = set_smem_limit<PRO, EPI, 8>()) ||
        (r = set_smem_limit<PRO, EPI, 10>()) || (r = set_smem_limit<PRO, EPI, 12>()) ||
        (r = set_smem_limit<PRO, EPI, 16>()))
        return r;
    return 0;
}

int prepare_other_kernels();  // attention and the small kernels (defined after them)

// Raises every kernel's dynamic shared-memory limit on the current device.
// Runs once per device (outside any stream capture: the first launch of each
// kind on a device should not be captured); later calls cost one
// cudaGetDevice and an atomic load.
int prepare_kernels() {
    const int dev = current_device();
    if (dev < 0) return H4B_EUNSUPPORTED;
    if (g_devices[dev].prepared.load(std::memory_order_acquire)) return 0;
    std::lock_guard<std::mutex> lock(g_prepare_mutex);
    if (g_devices[dev].prepared.load(std::memory_order_relaxed)) return 0;
    int r = 0;
    if ((r = set_smem_limits<PRO_INT8, EPI_STORE>()) || (r = set_smem_limits<PRO_QUANT, EPI_STORE>()) ||
        (r = set_smem_limits<PRO_RMSNORM, EPI_STORE>()) || (r = set_smem_limits<PRO_QUANT_ABSMAX, EPI_RESIDUAL>()) ||
        (r = set_smem_limits<PRO_QUANT_ABSMAX, EPI_STORE>()) ||
        (r = set_smem_limits<PRO_RMSNORM, EPI_SWIGLU>()) || (r = set_smem_limits<PRO_RMSNORM, EPI_ARGMAX>()))
        return r;
    if ((r = prepare_other_kernels())) return r;
    sm_count();
    g_devices[dev].prepared.store(true, std::memory_order_release);
    return 0;
}

template <int PRO, int EPI, int SLOTS>
static int launch_t(const GemvArgs& a, const GemvPlan& p, cudaStream_t stream, bool pdl) {
    auto kernel = gemv_kernel<PRO, EPI, SLOTS>;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    H4B_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, a));
    return 0;
}

template <int PRO, int EPI>
static int launch_slots(const GemvArgs& a, const GemvPlan& p, cudaStream_t s, bool pdl) {
    switch (p.slots) {
        case 1: return launch_t<PRO, EPI, 1>(a, p, s, pdl);
        case 2: return launch_t<PRO, EPI, 2>(a, p, s, pdl);
        case 3: return launch_t<PRO, EPI, 3>(a, p, s, pdl);
        case 4: return launch_t<PRO, EPI, 4>(a, p, s, pdl);
        case 6: return launch_t<PRO, EPI, 6>(a, p, s, pdl);
        case 8: return launch_t<PRO, EPI, 8>(a, p, s, pdl);
        case 10: return launch_t<PRO, EPI, 10>(a, p, s, pdl);
        case 12: return launch_t<PRO, EPI, 12>(a, p, s, pdl);
        case 16: return launch_t<PRO, EPI, 16>(a, p, s, pdl);
        default: return H4B_EUNSUPPORTED;
    }
}

// The (prologue, epilogue) pairs the decode path and the C ABI use.
int launch_gemv(int pro, int epi, GemvArgs a, cudaStream_t stream, bool pdl) {
    {
        const int prc = prepare_kernels();
        if (prc) return prc;
    }
    const int align = (epi == EPI_SWIGLU) ? 2 * kSwigluBlock : 1;
    GemvPlan p;
    const int rc = plan_gemv(a.rows, a.width, align, &p);
    if (rc) return rc;
    if (reinterpret_cast<uintptr_t>(a.w) & 15) return H4B_EINVAL;
    a.row_align = align;
    a.tile_rows = p.tile_rows;
    a.stages = p.stages;
    a.rows_cap = p.rows_cap;
    if (pro == PRO_INT8 && epi == EPI_STORE) return launch_slots<PRO_INT8, EPI_STORE>(a, p, stream, pdl);
    if (pro == PRO_QUANT && epi == EPI_STORE) return launch_slots<PRO_QUANT, EPI_STORE>(a, p, stream, pdl);
    if (pro == PRO_RMSNORM && epi == EPI_STORE) return launch_slots<PRO_RMSNORM, EPI_STORE>(a, p, stream, pdl);
    if (pro == PRO_QUANT_ABSMAX && epi == EPI_RESIDUAL)
        return launch_slots<PRO_QUANT_ABSMAX, EPI_RESIDUAL>(a, p, stream, pdl);
    if (pro == PRO_QUANT_ABSMAX && epi == EPI_STORE)
        return launch_slots<PRO_QUANT_ABSMAX, EPI_STORE>(a, p, stream, pdl);
    if (pro == PRO_RMSNORM && epi == EPI_SWIGLU) return launch_slots<PRO_RMSNORM, EPI_SWIGLU>(a, p, stream, pdl);
    if (pro == PRO_RMSNORM && epi == EPI_ARGMAX) return launch_slots<PRO_RMSNORM, EPI_ARGMAX>(a, p, stream, pdl);
    return H4B_EUNSUPPORTED;
}

}  // namespace h4b

// ---------------------------------------------------------------------------
// C ABI (declared in include/harsh4b_b200.h)

extern "C" int h4b_int4_i8_gemv(const int8_t* x, const uint8_t* weights, const float* scales,
                                float activation_scale, float* output, int32_t* acc, int rows, int width,
                                void* stream) {
    if (!x || !weights || !scales || !output) return H4B_EINVAL;
    if (reinterpret_cast<uintptr_t>(x) & 7) return H4B_EINVAL;
    h4b::GemvArgs a = {};
    a.w = weights; a.wscale = scales; a.rows = rows; a.width = width;
    a.x8 = x; a.act_scale = activation_scale; a.out = output; a.acc_out = acc;
    return h4b::launch_gemv(h4b::PRO_INT8, h4b::EPI_STORE, a, static_cast<cudaStream_t>(stream), false);
}

extern "C" int h4b_int4_gemv_fused_quant(const float* values, const uint8_t* weights, const float* scales,
                                         float* output, int32_t* acc, float* act_scale_out, int rows,
                                         int width, void* stream) {
    if (!values || !weights || !scales || !output) return H4B_EINVAL;
    if (reinterpret_cast<uintptr_t>(values) & 15) return H4B_EINVAL;
    h4b::GemvArgs a = {};
    a.w = weights; a.wscale = scales; a.rows = rows; a.width = width;
    a.xin = values; a.out = output; a.acc_out = acc; a.act_scale_out = act_scale_out;
    return h4b::launch_gemv(h4b::PRO_QUANT, h4b::EPI_STORE, a, static_cast<cudaStream_t>(stream), false);
}

extern "C" int h4b_int4_gemv_fused_quant_ex(const float* values, const uint8_t* weights, const float* scales,
                                            float* output, int32_t* acc, float* act_scale_out, int rows, int width,
                                            int flags, void* stream) {
    if (!values || !weights || !scales || !output || (flags & ~H4B_LAUNCH_PDL)) return H4B_EINVAL;
    if (reinterpret_cast<uintptr_t>(values) & 15) return H4B_EINVAL;
    h4b::GemvArgs a = {};
    a.w = weights; a.wscale = scales; a.rows = rows; a.width = width;
    a.xin = values; a.out = output; a.acc_out = acc; a.act_scale_out = act_scale_out;
    return h4b::launch_gemv(h4b::PRO_QUANT, h4b::EPI_STORE, a, static_cast<cudaStream_t>(stream),
                            (flags & H4B_LAUNCH_PDL) != 0);
}

// Quantisation with a given absmax (a device scalar, e.g. the max over the
// ranks of a tensor-parallel group) fused with the GEMV; writes the int32
// row sums (and the fp32 rows when `output` is not null).
extern "C" int h4b_int4_gemv_absmax(const float* values, const float* absmax, const uint8_t* weights,
                                    const float* scales, float* output, int32_t* acc, int rows, int width,
                                    void* stream) {
    if (!values || !absmax || !weights || !scales || !acc) return H4B_EINVAL;
    if (reinterpret_cast<uintptr_t>(values) & 15) return H4B_EINVAL;
    h4b::GemvArgs a = {};
    a.w = weights; a.wscale = scales; a.rows = rows; a.width = width;
    a.xin = values; a.absmax_in = absmax; a.out = output; a.acc_out = acc;
    return h4b::launch_gemv(h4b::PRO_QUANT_ABSMAX, h4b::EPI_STORE, a, static_cast<cudaStream_t>(stream), false);
}
