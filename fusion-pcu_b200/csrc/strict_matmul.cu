// strict_matmul.cu -- ordered-K checked F32/F64 MatMul for sm_100a.
//
// Semantics (paths relative to the Fusion-PCU checkout): every output cell folds k = 0..K-1 in
// increasing order from +0, rounding the multiply, then the add, each checked under the
// node's underflow policy (Crates/core/dialect/tensor/reference/strict_matmul/strict_matmul.rs:22-73,
// CPU order Crates/backends/cpu/prepared_tensor/execution/execution.rs:243-281).  The first
// fault is the lowest event (cell*K + k)*2 + {Multiply 0, Add 1}
// (Crates/core/dialect/tensor/fault_domain/fault_domain.rs:131-142), recorded with atomicMin as
// the reference kernel does (Crates/backends/cuda/tensor/strict_matmul/strict_matmul.rs:253-256).
//
// B200 design.  The strict contract forbids FMA and reassociation, so tensor cores cannot be
// used: the kernel is bound by the FP32 (FP64) CUDA-core issue rate, one FMUL and one FADD
// per (cell, k).  Everything else is organised to keep other instructions off the issue ports:
//   * TMA (cp.async.bulk.tensor, no multicast) stages A and B tiles into a 4-stage shared
//     memory ring driven by one producer thread and mbarriers; K-major tiles use the 128-byte
//     swizzle so the consumers' 16-byte fragment loads are bank-conflict free.
//   * 256 consumer threads each own an 8x8 (F32) or 8x4 (F64) register block of cells and run
//     __fmul_rn/__fadd_rn on 16-byte shared-memory fragments: 4 LDS.128 per 128 FP32 ops.
//   * Fault detection costs nothing in the loop.  Overflow and invalid operands are sticky
//     through IEEE add/multiply, so a finite final sum proves neither happened.  A tiny
//     (underflowing) product is only possible when the smallest nonzero operand exponents of
//     the cell's row of op(A) and column of op(B) add up below the format's limit; a prescan
//     kernel computes those minima once per call.  Cells that fail either test re-walk their
//     K range with the exact checked law (checked_law.cuh) to find the first fault; all other
//     cells are bit-identical to the law because no step faulted.
//   * Shapes whose strides or base addresses TMA cannot describe use a plain tiled kernel
//     with the same epilogue.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "pcu_b200.h"
#include "provider.h"

// Tuning knobs (defaults are the measured best; override with -D for sweeps).
#ifndef PCU_MM_UNROLL_F32
#define PCU_MM_UNROLL_F32 2
#endif
#ifndef PCU_MM_UNROLL_F64
#define PCU_MM_UNROLL_F64 8
#endif
#ifndef PCU_MM_LOOKAHEAD
#define PCU_MM_LOOKAHEAD 2
#endif

namespace pcu {

constexpr int kMaxPeers = 7;  // up to 8 GPUs of one node

// Elementwise stages fused into the MatMul's epilogue (pcu_b200_strict_matmul_epilogue): stage s
// takes the previous value (the MatMul's result for stage 0) and, for a checked binary op or
// ReLU-backward, one more operand laid out like the output (or one uniform element), writes its
// own output and records its first fault, with the element-index events of an elementwise
// node, in its own status word.  A cell whose MatMul (or earlier stage) faulted runs no later
// stage: that node's fault is reported before any of theirs.
constexpr int kMaxEpilogue = PCU_B200_EPILOGUE_MAX;
template <typename T> struct EpilogueParams {
    int count;
    int op[kMaxEpilogue];            // PCU_B200_ADD..DIV, PCU_B200_EPILOGUE_RELU, _RELU_BACKWARD
    const T *operand[kMaxEpilogue];  // binary op or ReLU-backward: the other argument
    int uniform[kMaxEpilogue];       // the operand is one element, used for every cell
    int operand_left[kMaxEpilogue];  // the operand is the left argument: op(operand, value)
    T *out[kMaxEpilogue];
    unsigned long long *status[kMaxEpilogue];
};

template <typename T> struct MatmulParams {
    const T *left;
    const T *right;
    T *out;
    uint64_t rows, inner, columns, left_stride, right_stride;
    int transpose_left, transpose_right, policy, threshold;
    const int *row_minexp;  // null when no product can be rejected for underflow (gradual policy)
    const int *col_minexp;
    unsigned long long *status;
    int vector_out;  // out is 16-byte aligned and columns is a multiple of the 16-byte vector
    ChainGuard guard;  // the node's stage of a guarded chain (empty when not guarded)
    // A row block of a row-sharded product: every output element also goes to the same place in
    // each peer's copy of C (peer memory mapped into this process), and events are shifted by
    // event_base (the block's first cell times inner times 2) to the whole product's ordinals.
    T *peer_out[kMaxPeers];
    int npeers;
    unsigned long long event_base;
    // Write-after-read order of the peer stores (the "entered" words of the peer buffers):
    // every CTA stores `epoch` into signal[q], this rank's word in peer q's flag block, when it
    // starts; before its first peer store it waits until await_[q], peer q's word in this rank's
    // block, has reached `epoch`, i.e. until peer q's kernel of the same call has started and so
    // every earlier kernel on that peer's stream (the readers of its C) has finished.
    unsigned long long *signal[kMaxPeers];
    const unsigned long long *await_[kMaxPeers];
    unsigned long long epoch;
    // CTA schedule: the launch covers linear tiles [tile_first, tile_first + gridDim.x / split)
    // of a tiles_m x tiles_n grid of (16 * Tile<T>::TM) x BN tiles, visited in the grouped
    // order; with split 2 each CTA computes one half (BM rows) of a tile.
    unsigned tiles_m, tiles_n, tile_first;
    int split;
    EpilogueParams<T> epi;  // fused elementwise stages (count 0: none)
};

// The fused stages of one output cell (out of line: only products with an epilogue reach it).
template <typename T> __device__ __noinline__ void epilogue_cell(const MatmulParams<T> &p, uint64_t idx, T v) {
    for (int s = 0; s < p.epi.count; ++s) {
        const int op = p.epi.op[s];
        T o;
        unsigned kind;
        if (op == PCU_B200_EPILOGUE_RELU) {
            kind = checked_relu<T>(v, p.policy, o);
        } else {
            const T w = p.epi.operand[s][p.epi.uniform[s] ? 0 : idx];
            const T a = p.epi.operand_left[s] ? w : v, b = p.epi.operand_left[s] ? v : w;
            kind = op == PCU_B200_EPILOGUE_RELU_BACKWARD ? checked_relu_backward<T>(a, b, p.policy, o)
                                                         : checked_binary<T>(op, a, b, p.policy, o);
        }
        if (kind) {
            record_fault(p.epi.status[s], idx, kind);
            return;
        }
        p.epi.out[s][idx] = o;
        v = o;
    }
}

// an output element (or 16-byte vector): this device's C and the first np peers' copies, then
// the fused stages, if any
template <typename T, typename X>
__device__ __forceinline__ void put_out(const MatmulParams<T> &p, int np, uint64_t idx, X v) {
    *reinterpret_cast<X *>(p.out + idx) = v;
    for (int q = 0; q < np; ++q) *reinterpret_cast<X *>(p.peer_out[q] + idx) = v;
    if (p.epi.count) {
        constexpr int kCells = sizeof(X) / sizeof(T);
#pragma unroll
        for (int q = 0; q < kCells; ++q) epilogue_cell<T>(p, idx + q, reinterpret_cast<const T *>(&v)[q]);
    }
}

// Every CTA of a row-sharded call announces, in each peer's flag block, that this rank has
// entered call `epoch` (one thread; plain system-scope stores over NVLink).
template <typename T> __device__ __forceinline__ void announce_entry(const MatmulParams<T> &p) {
    if (!p.npeers || threadIdx.x != 0) return;
    for (int q = 0; q < p.npeers; ++q)
        asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p.signal[q]), "l"(p.epoch) : "memory");
}

__device__ __forceinline__ unsigned long long load_acquire_sys(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Thread 0: how many peers this CTA may store into.  It waits (bounded) until every peer has
// entered this call; a peer that has not within kPeerWaitLimitNs gets no stores, and the
// status word records kWatchdog (event 0), which also tells later CTAs not to wait again.
template <typename T> __device__ __noinline__ int peers_entered(const MatmulParams<T> &p) {
    constexpr unsigned long long kGaveUp = (0ull << 3) | kWatchdog;
    const unsigned long long t0 = global_ns();
    for (int q = 0; q < p.npeers; ++q) {
        while (load_acquire_sys(p.await_[q]) < p.epoch) {
            if (read_status(p.status) == kGaveUp || global_ns() - t0 > kPeerWaitLimitNs) {
                record_fault(p.status, 0, kWatchdog);
                return 0;
            }
            __nanosleep(256);
        }
    }
    return p.npeers;
}

// "no nonzero finite element" marker of the exponent prescan (also the memset byte pattern)
constexpr int kNoExponent = 0x10101010;

template <typename T> __device__ __forceinline__ int min_exponent_of(T x);

template <> __device__ __forceinline__ int min_exponent_of<float>(float x) {
    uint32_t u = __float_as_uint(x);
    uint32_t e = (u >> 23) & 0xffu;
    if (e == 0xffu || (u << 1) == 0) return kNoExponent;
    if (e) return (int)e - 127;
    return (31 - __clz(u & 0x7fffffu)) - 149;
}

template <> __device__ __forceinline__ int min_exponent_of<double>(double x) {
    uint64_t u = (uint64_t)__double_as_longlong(x);
    uint32_t e = (uint32_t)((u >> 52) & 0x7ffu);
    if (e == 0x7ffu || (u << 1) == 0) return kNoExponent;
    if (e) return (int)e - 1023;
    return (63 - __clzll((long long)(u & 0x000fffffffffffffull))) - 1074;
}

// min exponent along each row of a rows x cols row-major matrix (one warp per row)
template <typename T>
__global__ void __launch_bounds__(256) minexp_rows_kernel(const T *x, uint64_t rows, uint64_t cols, uint64_t ld,
                                                          int *out, ChainGuard guard) {
    if (!chain_admits(guard)) return;
    const uint64_t warps = (uint64_t)gridDim.x * (blockDim.x / 32);
    const uint64_t warp = (uint64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    for (uint64_t r = warp; r < rows; r += warps) {
        const T *row = x + r * ld;
        int m = kNoExponent;
        for (uint64_t c = lane; c < cols; c += 32) m = min(m, min_exponent_of<T>(__ldg(row + c)));
#pragma unroll
        for (int o = 16; o; o >>= 1) m = min(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) out[r] = m;
    }
}

// min exponent down each column; blockIdx.y takes a slab of rows, atomicMin merges slabs
template <typename T>
__global__ void __launch_bounds__(256) minexp_cols_kernel(const T *x, uint64_t rows, uint64_t cols, uint64_t ld,
                                                          uint64_t rows_per_slab, int *out, ChainGuard guard) {
    if (!chain_admits(guard)) return;
    const uint64_t c = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cols) return;
    const uint64_t r0 = (uint64_t)blockIdx.y * rows_per_slab;
    const uint64_t r1 = r0 + rows_per_slab < rows ? r0 + rows_per_slab : rows;
    int m = kNoExponent;
    for (uint64_t r = r0; r < r1; ++r) m = min(m, min_exponent_of<T>(__ldg(x + r * ld + c)));
    if (m != kNoExponent) atomicMin(out + c, m);
}

template <typename T>
__device__ __forceinline__ T load_a(const MatmulParams<T> &p, uint64_t r, uint64_t k) {
    return p.transpose_left ? p.left[k * p.left_stride + r] : p.left[r * p.left_stride + k];
}

template <typename T>
__device__ __forceinline__ T load_b(const MatmulParams<T> &p, uint64_t k, uint64_t c) {
    return p.transpose_right ? p.right[c * p.right_stride + k] : p.right[k * p.right_stride + c];
}

// Exact ordered walk of one cell with the checked law; records its first fault.
template <typename T>
__device__ __noinline__ void exact_cell(const MatmulParams<T> &p, int np, uint64_t r, uint64_t c) {
    const uint64_t cell = r * p.columns + c;
    const uint64_t base = p.event_base + cell * p.inner * 2;
    if (fault_precedes(p.status, base)) return;
    T acc = T(0);
    for (uint64_t k = 0; k < p.inner; ++k) {
        T prod;
        unsigned kind = checked_mul<T>(load_a(p, r, k), load_b(p, k, c), p.policy, prod);
        if (kind) { record_fault(p.status, base + 2 * k, kind); return; }
        kind = checked_add<T>(acc, prod, p.policy, acc);
        if (kind) { record_fault(p.status, base + 2 * k + 1, kind); return; }
        if ((k & 1023) == 1023 && fault_precedes(p.status, base + 2 * k)) return;
    }
    put_out<T, T>(p, np, cell, acc);
}

// Does the fast result of cell (r, c) need the exact walk?
template <typename T>
__device__ __forceinline__ bool needs_exact(const MatmulParams<T> &p, T acc, int rmin, int cmin) {
    return nonfinite_bits<T>(Fmt<T>::bits(acc)) || (p.row_minexp && rmin + cmin < p.threshold);
}

// ------------------------------------------------------------------ TMA / mbarrier helpers
__device__ __forceinline__ uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded wait: false after kWaitLimitNs (the caller reports kWatchdog).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    for (;;) {
#pragma unroll 1
        for (int i = 0; i < 64; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (global_ns() - t0 > kWaitLimitNs) return false;
    }
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
            "r"(smem_addr(dst)),
        "l"(map), "r"(smem_addr(bar)), "r"(x), "r"(y)
        : "memory");
}

template <typename T> struct Tile;
// GROUP_UNROLL: 16-byte K groups folded per loop iteration (measured best on B200:
// 2 for binary32, whose group body is 512 FP instructions; 8 for binary64, 128 per group).
template <> struct Tile<float> {
    static constexpr int TM = 8, TN = 8, BK = 32, STAGES = 4, GROUP_UNROLL = PCU_MM_UNROLL_F32;
};
template <> struct Tile<double> {
    static constexpr int TM = 8, TN = 4, BK = 16, STAGES = 4, GROUP_UNROLL = PCU_MM_UNROLL_F64;
};

template <typename T, int V> struct SVec;
template <> struct SVec<float, 4> { using type = float4; };
template <> struct SVec<double, 2> { using type = double2; };

// TM_ rows of cells per thread: Tile<T>::TM for whole tiles, half of it for the half tiles that
// fill the last wave of a launch (the tile's BM rows then take two CTAs).
template <typename T, int TM_ = Tile<T>::TM> struct TileShape {
    static constexpr int V = 16 / sizeof(T);  // elements per 16-byte fragment
    static constexpr int TM = TM_, TN = Tile<T>::TN, BK = Tile<T>::BK, STAGES = Tile<T>::STAGES;
    static constexpr int BM = 16 * TM, BN = 16 * TN;
    static constexpr int A_BYTES = BM * BK * (int)sizeof(T);
    static constexpr int B_BYTES = BN * BK * (int)sizeof(T);
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 2 * STAGES * 8 + 1024;  // + barriers + align slack
    static_assert(BK * sizeof(T) == 128, "K-major tiles are one 128-byte swizzle row per M/N index");
};

// Eight warps, two per SM sub-partition: a ninth (producer) warp would put three warps on one
// sub-partition and cap every thread at 168 registers.  Thread 0 issues the TMA copies instead.
constexpr int kConsumerWarps = 8;
constexpr int kThreads = kConsumerWarps * 32;
constexpr unsigned kGroupRows = 8;  // tile rows per group of the CTA order
// Stages in flight beyond the one being folded.  Thread 0 refills the slot of stage kt-2 while
// folding stage kt, so it practically never waits for a slower warp to release a slot.
constexpr int kLookahead = PCU_MM_LOOKAHEAD;
static_assert(kLookahead >= 1 && kLookahead < 4, "lookahead must leave a slot free");

// A_KMAJOR: op(A) rows are contiguous in k (left not transposed).
// B_KMAJOR: op(B) columns are contiguous in k (right transposed).
// TMv: rows of cells per thread (Tile<T>::TM, or half of it for half tiles).
template <typename T, bool A_KMAJOR, bool B_KMAJOR, int TMv>
__global__ void __launch_bounds__(kThreads, 1)
    strict_matmul_tma_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                             const __grid_constant__ MatmulParams<T> p) {
    using S = TileShape<T, TMv>;
    constexpr int V = S::V, TM = S::TM, TN = S::TN, BK = S::BK, BM = S::BM, BN = S::BN, STAGES = S::STAGES;
    using VT = typename SVec<T, V>::type;
    using F = Fmt<T>;

    if (!chain_admits(p.guard)) return;  // the whole CTA, before any barrier or copy
    announce_entry(p);
    extern __shared__ unsigned char smem_raw[];
    const uintptr_t base = (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023);
    T *const tiles = reinterpret_cast<T *>(base);
    uint64_t *const full = reinterpret_cast<uint64_t *>(base + STAGES * S::STAGE_BYTES);
    uint64_t *const empty = full + STAGES;
    __shared__ int abort_flag;
    __shared__ int peers_ok;

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    // Tiles in groups of kGroupRows tile rows, column by column inside a group: the CTAs resident
    // at once share a few A row panels and B column panels, which stay in L2 while they are read.
    uint64_t m0, n0;
    {
        const unsigned tiles_n = p.tiles_n, tiles_m = p.tiles_m;
        const unsigned id = p.tile_first + blockIdx.x / (unsigned)p.split;  // launch order
        const unsigned first_m = id / (kGroupRows * tiles_n) * kGroupRows;
        const unsigned rows_here = min((unsigned)kGroupRows, tiles_m - first_m);
        const unsigned in_group = id - first_m * tiles_n;
        m0 = (uint64_t)(first_m + in_group % rows_here) * (BM * p.split) + (uint64_t)(blockIdx.x % p.split) * BM;
        n0 = (uint64_t)(in_group / rows_here) * BN;
    }
    const int KT = (int)((p.inner + BK - 1) / BK);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        abort_flag = 0;
    }
    __syncthreads();

    // Thread 0 only: copy stage `kt` into its slot once every warp has released the slot.
    int issued = 0;
    auto issue = [&](int kt) -> bool {
        const int s = kt % STAGES;
        if (!mbar_wait(&empty[s], ((kt / STAGES) & 1) ^ 1)) {
            record_fault(p.status, 0, kWatchdog);
            abort_flag = 1;
            return false;
        }
        T *sa = tiles + (size_t)s * (S::STAGE_BYTES / sizeof(T));
        T *sb = sa + S::A_BYTES / sizeof(T);
        mbar_expect_tx(&full[s], S::STAGE_BYTES);
        const int k0 = kt * BK;
        if (A_KMAJOR) tma_load_2d(sa, &map_a, &full[s], k0, (int)m0);
        else tma_load_2d(sa, &map_a, &full[s], (int)m0, k0);
        if (B_KMAJOR) tma_load_2d(sb, &map_b, &full[s], k0, (int)n0);
        else tma_load_2d(sb, &map_b, &full[s], (int)n0, k0);
        ++issued;
        return true;
    };
    if (threadIdx.x == 0)
        for (int kt = 0; kt < kLookahead && kt < KT; ++kt)
            if (!issue(kt)) break;

    // -------------------------------------------------------------------- consumers
    const int ty = (warp >> 1) * 4 + (lane >> 3);  // 0..15 along M
    const int tx = (warp & 1) * 8 + (lane & 7);    // 0..15 along N

    // M (N) offsets of this thread's cells inside the tile.  K-major tiles use a stride of 16
    // (rows ty, ty+16, ...) so the 128-byte swizzle spreads a warp over distinct banks;
    // MN-major tiles use runs of V contiguous elements for 16-byte fragment loads.
    auto row_of = [&](int i) -> int { return A_KMAJOR ? ty + 16 * i : (i / V) * (16 * V) + ty * V + (i % V); };
    auto col_of = [&](int j) -> int { return B_KMAJOR ? tx + 16 * j : (j / V) * (16 * V) + tx * V + (j % V); };

    T acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = T(0);

    int kt = 0;
    for (; kt < KT; ++kt) {
        const int s = kt % STAGES;
        if (threadIdx.x == 0 && kt + kLookahead < KT && !*(volatile int *)&abort_flag) issue(kt + kLookahead);
        __syncwarp();
        if (!mbar_wait(&full[s], (kt / STAGES) & 1)) {
            record_fault(p.status, 0, kWatchdog);
            abort_flag = 1;
            break;
        }
        const T *sa = tiles + (size_t)s * (S::STAGE_BYTES / sizeof(T));
        const T *sb = sa + S::A_BYTES / sizeof(T);
        // One group = V k-steps of 16-byte fragments; a stage holds BK / V = 8 groups.
        auto load_group = [&](int g, T (&a)[TM][V], T (&b)[V][TN]) {
            if (A_KMAJOR) {
                const int chunk = g ^ (ty & 7);
#pragma unroll
                for (int i = 0; i < TM; ++i) {
                    VT v = *reinterpret_cast<const VT *>(sa + row_of(i) * BK + chunk * V);
                    const T *e = reinterpret_cast<const T *>(&v);
#pragma unroll
                    for (int kv = 0; kv < V; ++kv) a[i][kv] = e[kv];
                }
            } else {
#pragma unroll
                for (int kv = 0; kv < V; ++kv)
#pragma unroll
                    for (int ig = 0; ig < TM / V; ++ig) {
                        VT v = *reinterpret_cast<const VT *>(sa + (g * V + kv) * BM + ig * 16 * V + ty * V);
                        const T *e = reinterpret_cast<const T *>(&v);
#pragma unroll
                        for (int q = 0; q < V; ++q) a[ig * V + q][kv] = e[q];
                    }
            }
            if (B_KMAJOR) {
                const int chunk = g ^ (tx & 7);
#pragma unroll
                for (int j = 0; j < TN; ++j) {
                    VT v = *reinterpret_cast<const VT *>(sb + col_of(j) * BK + chunk * V);
                    const T *e = reinterpret_cast<const T *>(&v);
#pragma unroll
                    for (int kv = 0; kv < V; ++kv) b[kv][j] = e[kv];
                }
            } else {
#pragma unroll
                for (int kv = 0; kv < V; ++kv)
#pragma unroll
                    for (int jg = 0; jg < TN / V; ++jg) {
                        VT v = *reinterpret_cast<const VT *>(sb + (g * V + kv) * BN + jg * 16 * V + tx * V);
                        const T *e = reinterpret_cast<const T *>(&v);
#pragma unroll
                        for (int q = 0; q < V; ++q) b[kv][jg * V + q] = e[q];
                    }
            }
        };
        // k ascending inside the group: kv is the outer loop, so every cell sees its K in order
        auto fold_group = [&](const T (&a)[TM][V], const T (&b)[V][TN]) {
#pragma unroll
            for (int kv = 0; kv < V; ++kv)
#pragma unroll
                for (int i = 0; i < TM; ++i)
#pragma unroll
                    for (int j = 0; j < TN; ++j) acc[i][j] = F::add(acc[i][j], F::mul(a[i][kv], b[kv][j]));
        };
        // Unrolling all BK / V groups of a stage makes the body larger than the instruction
        // cache (measured: the no_instruction stall dominates); Tile<T>::GROUP_UNROLL groups
        // per loop iteration keep it resident.
        constexpr int kUnroll = Tile<T>::GROUP_UNROLL;
#pragma unroll kUnroll
        for (int g = 0; g < BK / V; ++g) {
            T a[TM][V], b[V][TN];
            load_group(g, a, b);
            fold_group(a, b);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    // Peer stores wait until every peer has entered this call (row-sharded form only).
    if (threadIdx.x == 0) peers_ok = p.npeers ? peers_entered(p) : 0;
    // Never leave the CTA with a bulk copy still writing into its shared memory: after a
    // watchdog abort thread 0 waits (bounded) for every copy it issued but nobody folded.
    __syncthreads();
    if (*(volatile int *)&abort_flag) {
        if (threadIdx.x == 0)
            for (int t = kt; t < issued; ++t)
                if (!mbar_wait(&full[t % STAGES], (t / STAGES) & 1)) break;
        return;
    }

    // -------------------------------------------------------------------- epilogue
    int rmin[TM], cmin[TN];
#pragma unroll
    for (int i = 0; i < TM; ++i) {
        const uint64_t r = m0 + row_of(i);
        rmin[i] = (p.row_minexp && r < p.rows) ? p.row_minexp[r] : 0;
    }
#pragma unroll
    for (int j = 0; j < TN; ++j) {
        const uint64_t c = n0 + col_of(j);
        cmin[j] = (p.col_minexp && c < p.columns) ? p.col_minexp[c] : 0;
    }
    const bool vec_store = !B_KMAJOR && p.vector_out;
    const int np = peers_ok;
#pragma unroll
    for (int i = 0; i < TM; ++i) {
        const uint64_t r = m0 + row_of(i);
        if (r >= p.rows) continue;
        if (vec_store) {
#pragma unroll
            for (int jg = 0; jg < TN / V; ++jg) {
                const uint64_t c = n0 + col_of(jg * V);
                if (c >= p.columns) continue;
                bool exact = false;
#pragma unroll
                for (int q = 0; q < V; ++q) exact |= needs_exact(p, acc[i][jg * V + q], rmin[i], cmin[jg * V + q]);
                if (!exact) {
                    VT v;
                    T *e = reinterpret_cast<T *>(&v);
#pragma unroll
                    for (int q = 0; q < V; ++q) e[q] = acc[i][jg * V + q];
                    put_out<T, VT>(p, np, r * p.columns + c, v);
                } else {
#pragma unroll
                    for (int q = 0; q < V; ++q) {
                        if (needs_exact(p, acc[i][jg * V + q], rmin[i], cmin[jg * V + q])) exact_cell(p, np, r, c + q);
                        else put_out<T, T>(p, np, r * p.columns + c + q, acc[i][jg * V + q]);
                    }
                }
            }
        } else {
#pragma unroll
            for (int j = 0; j < TN; ++j) {
                const uint64_t c = n0 + col_of(j);
                if (c >= p.columns) continue;
                if (needs_exact(p, acc[i][j], rmin[i], cmin[j])) exact_cell(p, np, r, c);
                else put_out<T, T>(p, np, r * p.columns + c, acc[i][j]);
            }
        }
    }
    // No fence after the peer stores: a kernel's writes, to peer memory as to any other, are
    // visible to everything ordered after its completion, and C is read only after the status
    // collective that follows this kernel on every rank.  A per-CTA system fence would hold the CTA
    // (and its SM) until its own stores had crossed NVLink behind those of every CTA finishing at
    // the same time, instead of letting them drain under the next wave's arithmetic.
}

// Plain tiled kernel for operands TMA cannot describe (unaligned base or stride): 16x16
// threads, one cell each, 16-deep K slabs through shared memory, same epilogue.
template <typename T>
__global__ void __launch_bounds__(256) strict_matmul_generic_kernel(const __grid_constant__ MatmulParams<T> p) {
    if (!chain_admits(p.guard)) return;  // the whole CTA
    announce_entry(p);
    using F = Fmt<T>;
    __shared__ T sa[16][17];
    __shared__ T sb[16][17];
    __shared__ int peers_ok;
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const uint64_t r = (uint64_t)blockIdx.y * 16 + ty, c = (uint64_t)blockIdx.x * 16 + tx;
    T acc = T(0);
    for (uint64_t k0 = 0; k0 < p.inner; k0 += 16) {
        const uint64_t ka = k0 + tx, kb = k0 + ty;
        const uint64_t ar = (uint64_t)blockIdx.y * 16 + ty, bc = (uint64_t)blockIdx.x * 16 + tx;
        sa[ty][tx] = (ar < p.rows && ka < p.inner) ? load_a(p, ar, ka) : T(0);
        sb[ty][tx] = (bc < p.columns && kb < p.inner) ? load_b(p, kb, bc) : T(0);
        __syncthreads();
        const int kk_end = (p.inner - k0) < 16 ? (int)(p.inner - k0) : 16;
        for (int kk = 0; kk < kk_end; ++kk) acc = F::add(acc, F::mul(sa[ty][kk], sb[kk][tx]));
        __syncthreads();
    }
    if (threadIdx.x == 0) peers_ok = p.npeers ? peers_entered(p) : 0;
    __syncthreads();
    const int np = peers_ok;
    if (r >= p.rows || c >= p.columns) return;
    const int rmin = p.row_minexp ? p.row_minexp[r] : 0;
    const int cmin = p.col_minexp ? p.col_minexp[c] : 0;
    if (needs_exact(p, acc, rmin, cmin)) exact_cell(p, np, r, c);
    else put_out<T, T>(p, np, r * p.columns + c, acc);
}

}  // namespace pcu

// ============================================================================ host side
namespace {

using namespace pcu;

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static std::once_flag once;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    std::call_once(once, [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

// 2-D tile map over a row-major matrix of `outer` rows x `inner_dim` elements with row
// stride `ld` elements; box = box_inner x box_outer elements.
template <typename T>
bool make_map(CUtensorMap *map, const T *base, uint64_t inner_dim, uint64_t outer, uint64_t ld, uint32_t box_inner,
              uint32_t box_outer, bool swizzle128) {
    auto encode = tensor_map_encoder();
    if (!encode) return false;
    if (!pcu_host::aligned(base, 16) || (ld * sizeof(T)) % 16 != 0) return false;
    if (inner_dim == 0 || outer == 0 || inner_dim >= (1ull << 31) || outer >= (1ull << 31)) return false;
    if (ld * sizeof(T) >= (1ull << 40)) return false;
    cuuint64_t dims[2] = {inner_dim, outer};
    cuuint64_t strides[1] = {ld * sizeof(T)};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estrides[2] = {1, 1};
    CUresult r = encode(map, sizeof(T) == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT64, 2,
                        const_cast<T *>(base), dims, strides, box, estrides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// One launch of `ctas` CTAs of the TMA kernel with TMv rows of cells per thread.
template <typename T, bool AK, bool BK, int TMv>
int launch_tma(const CUtensorMap &ma, const CUtensorMap &mb, const MatmulParams<T> &p, unsigned ctas,
               cudaStream_t stream) {
    using S = TileShape<T, TMv>;
    static std::mutex lock;
    static bool configured[64] = {false};
    int device = 0;
    cudaGetDevice(&device);
    {
        std::lock_guard<std::mutex> guard(lock);
        if (device >= 0 && device < 64 && !configured[device]) {
            cudaError_t e = cudaFuncSetAttribute(strict_matmul_tma_kernel<T, AK, BK, TMv>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM_BYTES);
            if (e != cudaSuccess) return pcu_host::set_cuda_error(e);
            configured[device] = true;
        }
    }
    strict_matmul_tma_kernel<T, AK, BK, TMv><<<ctas, kThreads, S::SMEM_BYTES, stream>>>(ma, mb, p);
    return pcu_host::launch_status();
}

// Split of a product's tiles into launches.  The TMA kernel runs one CTA per SM, so T tiles take
// ceil(T / SMs) waves; when the last wave would be at most half full, its R = T mod SMs tiles
// run instead as 2R half tiles in a second launch, which takes about half a wave's time (8192 x
// 8192 rows of 1024 per GPU: 512 tiles = 3 waves + 68 tiles on 148 SMs, so 3.5 wave times
// instead of 4).  Returns the number of whole tiles of the first launch.
inline uint64_t whole_tile_launch(uint64_t tiles, uint64_t sms) {
    if (tiles <= sms) return tiles;
    const uint64_t rem = tiles % sms;
    return (rem != 0 && 2 * rem <= sms) ? tiles - rem : tiles;
}

template <typename T, bool AK, bool BK>
int launch_tma_split(const CUtensorMap &ma, const CUtensorMap &ma_half, const CUtensorMap &mb, MatmulParams<T> p,
                     uint64_t whole, uint64_t tiles, ChainGuard tail_guard, cudaStream_t stream) {
    constexpr int TM = Tile<T>::TM;
    p.tile_first = 0;
    p.split = 1;
    if (whole) {
        int rc = launch_tma<T, AK, BK, TM>(ma, mb, p, (unsigned)whole, stream);
        if (rc) return rc;
        p.guard = tail_guard;
    }
    if (whole == tiles) return PCU_B200_OK;
    p.tile_first = (unsigned)whole;
    p.split = 2;
    return launch_tma<T, AK, BK, TM / 2>(ma_half, mb, p, (unsigned)(2 * (tiles - whole)), stream);
}

// The peers of a row-sharded call: their copies of C (this rank's rows), the flag words this
// rank announces its entry in, the flag words it waits on, and the call's number.
template <typename T> struct PeerSet {
    T *out[kMaxPeers];
    unsigned long long *signal[kMaxPeers];
    const unsigned long long *await_[kMaxPeers];
    int count = 0;
    unsigned long long epoch = 0;
};

template <typename T>
int run_matmul(int policy, const T *left, const T *right, T *out, uint64_t rows, uint64_t inner, uint64_t columns,
               uint64_t lda, uint64_t ldb, int tl, int tr, void *workspace, size_t workspace_bytes,
               unsigned long long *status, cudaStream_t stream, const ChainGuard &guard,
               const PeerSet<T> *peers = nullptr, unsigned long long event_base = 0,
               const EpilogueParams<T> *epi = nullptr) {
    MatmulParams<T> p{left,    right,   out,    rows,
                      inner,   columns, lda,    ldb,
                      tl,      tr,      policy, 0,
                      nullptr, nullptr, status, pcu_host::aligned(out, 16) && columns % (16 / sizeof(T)) == 0,
                      guard};
    p.npeers = peers ? peers->count : 0;
    for (int q = 0; q < p.npeers; ++q) {
        p.peer_out[q] = peers->out[q];
        p.signal[q] = peers->signal[q];
        p.await_[q] = peers->await_[q];
    }
    p.epoch = peers ? peers->epoch : 0;
    p.event_base = event_base;
    p.tiles_m = p.tiles_n = p.tile_first = 0;
    p.split = 1;
    p.epi = epi ? *epi : EpilogueParams<T>{};
    // the first kernel launched decides the stage's admission, the later ones follow it
    ChainGuard next = guard;
    auto take = [&]() {
        const ChainGuard g = next;
        next = chain_follow(next);
        return g;
    };
    if (policy != kPolicyGradual && inner > 0) {
        size_t need = pcu_b200_strict_matmul_workspace_size(rows, inner, columns);
        if (!workspace || workspace_bytes < need) return PCU_B200_ERROR_WORKSPACE;
        int *row_min = reinterpret_cast<int *>(workspace);
        int *col_min = reinterpret_cast<int *>(reinterpret_cast<char *>(workspace) + ((rows * 4 + 255) / 256) * 256);
        cudaError_t e = cudaMemsetAsync(workspace, 0x10, need, stream);
        if (e != cudaSuccess) return pcu_host::set_cuda_error(e);
        const int sms = pcu_host::sm_count();
        auto rows_pass = [&](const T *x, uint64_t r, uint64_t c, uint64_t ld, int *dst) {
            uint64_t blocks = (r + 7) / 8;
            if (blocks > (uint64_t)sms * 16) blocks = (uint64_t)sms * 16;
            minexp_rows_kernel<T><<<(unsigned)blocks, 256, 0, stream>>>(x, r, c, ld, dst, take());
        };
        auto cols_pass = [&](const T *x, uint64_t r, uint64_t c, uint64_t ld, int *dst) {
            uint64_t col_blocks = (c + 255) / 256;
            uint64_t slabs = ((uint64_t)sms * 8 + col_blocks - 1) / col_blocks;
            if (slabs > r) slabs = r;
            if (slabs > 65535) slabs = 65535;
            uint64_t per = (r + slabs - 1) / slabs;
            slabs = (r + per - 1) / per;
            minexp_cols_kernel<T><<<dim3((unsigned)col_blocks, (unsigned)slabs), 256, 0, stream>>>(x, r, c, ld, per,
                                                                                                 dst, take());
        };
        if (!tl) rows_pass(left, rows, inner, lda, row_min);
        else cols_pass(left, inner, rows, lda, row_min);
        if (!tr) cols_pass(right, inner, columns, ldb, col_min);
        else rows_pass(right, columns, inner, ldb, col_min);
        int rc = pcu_host::launch_status();
        if (rc) return rc;
        p.row_minexp = row_min;
        p.col_minexp = col_min;
        // A product below 2^(threshold) may be tiny (IEEE policy); under RejectSubnormalResult
        // every intermediate is a multiple of 2^(emin_a + emin_b - 2*frac), which must stay normal.
        const int frac = sizeof(T) == 4 ? 23 : 52;
        const int emin = sizeof(T) == 4 ? -126 : -1022;
        p.threshold = policy == kPolicyIeee ? emin : emin + 2 * frac;
    }
    p.guard = take();
    using S = TileShape<T>;
    using H = TileShape<T, Tile<T>::TM / 2>;
    CUtensorMap ma, ma_half, mb;
    bool tma = inner > 0;
    if (tma) {
        tma = tl ? make_map<T>(&ma, left, rows, inner, lda, S::BM, S::BK, false)
                 : make_map<T>(&ma, left, inner, rows, lda, S::BK, S::BM, true);
    }
    if (tma) {
        tma = tr ? make_map<T>(&mb, right, inner, columns, ldb, S::BK, S::BN, true)
                 : make_map<T>(&mb, right, columns, inner, ldb, S::BN, S::BK, false);
    }
    // An output of a few 128-wide tiles would leave most SMs idle (a 256 x 256 product is 4
    // CTAs); the 16 x 16-tile kernel spreads it over many CTAs instead.
    const uint64_t tiles_m = (rows + S::BM - 1) / S::BM, tiles_n = (columns + S::BN - 1) / S::BN;
    const uint64_t tiles = tiles_m * tiles_n;
    const uint64_t sms = (uint64_t)pcu_host::sm_count();
    if (tiles * 4 < sms) tma = false;
    if (tma && tiles < (1ull << 30)) {
        uint64_t whole = whole_tile_launch(tiles, sms);
        if (whole < tiles) {
            const bool half_map = tl ? make_map<T>(&ma_half, left, rows, inner, lda, H::BM, H::BK, false)
                                     : make_map<T>(&ma_half, left, inner, rows, lda, H::BK, H::BM, true);
            if (!half_map) whole = tiles;
        }
        p.tiles_m = (unsigned)tiles_m;
        p.tiles_n = (unsigned)tiles_n;
        const ChainGuard tail_guard = take();
        if (!tl && !tr) return launch_tma_split<T, true, false>(ma, ma_half, mb, p, whole, tiles, tail_guard, stream);
        if (!tl && tr) return launch_tma_split<T, true, true>(ma, ma_half, mb, p, whole, tiles, tail_guard, stream);
        if (tl && !tr) return launch_tma_split<T, false, false>(ma, ma_half, mb, p, whole, tiles, tail_guard, stream);
        return launch_tma_split<T, false, true>(ma, ma_half, mb, p, whole, tiles, tail_guard, stream);
    }
    if ((rows + 15) / 16 > 65535) return PCU_B200_ERROR_SIZE_OVERFLOW;
    dim3 grid((unsigned)((columns + 15) / 16), (unsigned)((rows + 15) / 16));
    strict_matmul_generic_kernel<T><<<grid, 256, 0, stream>>>(p);
    return pcu_host::launch_status();
}

}  // namespace

extern "C" size_t pcu_b200_strict_matmul_workspace_size(uint64_t rows, uint64_t inner, uint64_t columns) {
    (void)inner;
    return ((rows * 4 + 255) / 256) * 256 + ((columns * 4 + 255) / 256) * 256;
}

namespace {

template <typename T> EpilogueParams<T> epilogue_params(const pcu_b200_epilogue_stage *stages, int count) {
    EpilogueParams<T> e{};
    e.count = count;
    for (int i = 0; i < count; ++i) {
        e.op[i] = stages[i].op;
        e.operand[i] = static_cast<const T *>(stages[i].operand);
        e.uniform[i] = stages[i].operand_uniform != 0;
        e.operand_left[i] = stages[i].operand_left != 0;
        e.out[i] = static_cast<T *>(stages[i].out);
        e.status[i] = reinterpret_cast<unsigned long long *>(stages[i].status);
    }
    return e;
}

}  // namespace

int pcu::strict_matmul(int dtype, int policy, const void *left, const void *right, void *out, uint64_t rows,
                       uint64_t inner, uint64_t columns, uint64_t left_stride, uint64_t right_stride,
                       int transpose_left, int transpose_right, void *workspace, size_t workspace_bytes,
                       uint64_t *status, void *stream, const ChainGuard &guard,
                       const pcu_b200_epilogue_stage *stages, int stage_count) {
    if ((dtype != PCU_B200_F32 && dtype != PCU_B200_F64) || policy < 0 || policy > 2 || !status)
        return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (stage_count < 0 || stage_count > kMaxEpilogue || (stage_count && (!stages || guard.disp)))
        return PCU_B200_ERROR_INVALID_ARGUMENT;
    for (int i = 0; i < stage_count; ++i) {
        const pcu_b200_epilogue_stage &st = stages[i];
        const bool binary = st.op >= PCU_B200_ADD && st.op <= PCU_B200_DIV;
        if (!binary && st.op != PCU_B200_EPILOGUE_RELU && st.op != PCU_B200_EPILOGUE_RELU_BACKWARD)
            return PCU_B200_ERROR_INVALID_ARGUMENT;
        if (!st.status || ((rows && columns) && (!st.out || (st.op != PCU_B200_EPILOGUE_RELU && !st.operand))))
            return PCU_B200_ERROR_INVALID_ARGUMENT;
    }
    if (rows == 0 || columns == 0) return chain_decide_only(guard, pcu_host::as_stream(stream));
    if (!out || (inner > 0 && (!left || !right))) return PCU_B200_ERROR_INVALID_ARGUMENT;
    // left is rows x inner (or inner x rows); right is inner x columns (or columns x inner)
    const uint64_t left_row_len = transpose_left ? rows : inner;
    const uint64_t right_row_len = transpose_right ? inner : columns;
    if (inner > 0 && (left_stride < left_row_len || right_stride < right_row_len))
        return PCU_B200_ERROR_INVALID_ARGUMENT;
    // rows*columns*inner*2 <= 2^60 (strict_matmul.rs:121-127)
    unsigned __int128 events = (unsigned __int128)rows * columns;
    events *= (inner ? inner : 1);
    events *= 2;
    if (events > ((unsigned __int128)1 << 60)) return PCU_B200_ERROR_SIZE_OVERFLOW;
    auto *st = reinterpret_cast<unsigned long long *>(status);
    cudaStream_t s = pcu_host::as_stream(stream);
    if (dtype == PCU_B200_F32) {
        const EpilogueParams<float> epi = epilogue_params<float>(stages, stage_count);
        return run_matmul<float>(policy, (const float *)left, (const float *)right, (float *)out, rows, inner, columns,
                                 left_stride, right_stride, transpose_left != 0, transpose_right != 0, workspace,
                                 workspace_bytes, st, s, guard, nullptr, 0, stage_count ? &epi : nullptr);
    }
    const EpilogueParams<double> epi = epilogue_params<double>(stages, stage_count);
    return run_matmul<double>(policy, (const double *)left, (const double *)right, (double *)out, rows, inner,
                              columns, left_stride, right_stride, transpose_left != 0, transpose_right != 0,
                              workspace, workspace_bytes, st, s, guard, nullptr, 0, stage_count ? &epi : nullptr);
}

extern "C" int pcu_b200_strict_matmul_epilogue(int dtype, int policy, const void *left, const void *right, void *out,
                                               uint64_t rows, uint64_t inner, uint64_t columns, uint64_t left_stride,
                                               uint64_t right_stride, int transpose_left, int transpose_right,
                                               const pcu_b200_epilogue_stage *stages, int stage_count,
                                               void *workspace, size_t workspace_bytes, uint64_t *status,
                                               void *stream) {
    return pcu::strict_matmul(dtype, policy, left, right, out, rows, inner, columns, left_stride, right_stride,
                              transpose_left, transpose_right, workspace, workspace_bytes, status, stream,
                              ChainGuard{}, stages, stage_count);
}

extern "C" int pcu_b200_strict_matmul(int dtype, int policy, const void *left, const void *right, void *out,
                                      uint64_t rows, uint64_t inner, uint64_t columns, uint64_t left_stride,
                                      uint64_t right_stride, int transpose_left, int transpose_right,
                                      void *workspace, size_t workspace_bytes, uint64_t *status, void *stream) {
    return pcu::strict_matmul(dtype, policy, left, right, out, rows, inner, columns, left_stride, right_stride,
                              transpose_left, transpose_right, workspace, workspace_bytes, status, stream,
                              ChainGuard{});
}

// ============================================================================
// Strict MatMul for callers that cannot allocate device memory.
//
// Some callers of this library are handed only the operand, output and status buffers and have
// no way to obtain more device memory for the call: for example a plain C or FFI caller that is
// not the owner of the process's device allocator (in Fusion-PCU all device memory belongs to
// the Rust CudaMemoryResource pool), or a caller that must keep the call itself free of
// allocation.  pcu_b200_strict_matmul needs a workspace for the operand-exponent minima; this
// variant uses a fixed array of device memory that belongs to this library instead, and
// allocates nothing itself.
//
// The array is a file-scope __device__ variable, so every GPU that loads this library holds
// kStaticScratchBytes (about 257 KB) until the process exits.  Its limit is
// rows + columns <= kStaticScratchMaxExtent.  In host code the array's name is only a host-side
// handle, so the device address is looked up once per device with cudaGetSymbolAddress.
// ============================================================================
namespace {

constexpr uint64_t kStaticScratchMaxExtent = 65536;  // rows + columns
constexpr size_t kStaticScratchInts = kStaticScratchMaxExtent + 128;  // + 256-byte rounding of both halves
constexpr size_t kStaticScratchBytes = kStaticScratchInts * sizeof(int);

static __device__ __align__(256) int g_strict_matmul_scratch[kStaticScratchInts];

// The current context's unique id (cuCtxGetId through the runtime's driver entry point; the
// library does not link the driver at load time).  0 when it cannot be read.
unsigned long long current_context_id() {
    static std::once_flag once;
    static PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
    static PFN_cuCtxGetId_v12000 get_id = nullptr;
    std::call_once(once, [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(ptr);
        if (cudaGetDriverEntryPoint("cuCtxGetId", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(ptr);
    });
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS)
        return 0;
    return id;
}

// Device address of g_strict_matmul_scratch on the current device.  The first call on each
// device performs the lookup (cudaGetSymbolAddress, with that device current); later calls reuse
// it.  The cache is keyed on the device's context as well: after a device reset the module is
// loaded again, possibly elsewhere, so a new context gets a new lookup.
int static_scratch_address(void **address) {
    static std::mutex lock;
    static void *addresses[64] = {nullptr};
    static unsigned long long contexts[64] = {0};
    int device = 0;
    cudaError_t err = cudaGetDevice(&device);
    if (err != cudaSuccess) return pcu_host::set_cuda_error(err);
    if (device < 0 || device >= 64) return PCU_B200_ERROR_UNSUPPORTED;
    // 0 until this thread's runtime has made the device's context current; the lookup below does
    // that, so the id is read again after it
    const unsigned long long context = current_context_id();
    std::lock_guard<std::mutex> guard(lock);
    if (!addresses[device] || context == 0 || contexts[device] != context) {
        void *ptr = nullptr;
        err = cudaGetSymbolAddress(&ptr, g_strict_matmul_scratch);
        if (err != cudaSuccess) return pcu_host::set_cuda_error(err);
        addresses[device] = ptr;
        contexts[device] = current_context_id();
    }
    *address = addresses[device];
    return PCU_B200_OK;
}

}  // namespace

extern "C" int pcu_b200_strict_matmul_static_scratch(int dtype, int policy, const void *left, const void *right,
                                                     void *out, uint64_t rows, uint64_t inner, uint64_t columns,
                                                     uint64_t left_stride, uint64_t right_stride,
                                                     int transpose_left, int transpose_right, uint64_t *status,
                                                     void *stream) {
    if ((dtype != PCU_B200_F32 && dtype != PCU_B200_F64) || policy < 0 || policy > 2 || !status)
        return PCU_B200_ERROR_INVALID_ARGUMENT;
    // Only a call that computes products under a rejecting policy uses the exponent minima; the
    // others (empty shapes, inner == 0, AllowGradualUnderflow) need no scratch and no limit.
    const bool uses_scratch = policy != PCU_B200_ALLOW_GRADUAL_UNDERFLOW && rows > 0 && columns > 0 && inner > 0;
    if (!uses_scratch)
        return pcu_b200_strict_matmul(dtype, policy, left, right, out, rows, inner, columns, left_stride,
                                      right_stride, transpose_left, transpose_right, nullptr, 0, status, stream);
    if (rows > kStaticScratchMaxExtent || columns > kStaticScratchMaxExtent ||
        rows + columns > kStaticScratchMaxExtent)
        return PCU_B200_ERROR_WORKSPACE;
    void *scratch = nullptr;
    int rc = static_scratch_address(&scratch);
    if (rc != PCU_B200_OK) return rc;
    // pcu_b200_strict_matmul re-initialises the minima it needs on every call, so the contents
    // a previous call left in the shared array never leak into this one.
    return pcu_b200_strict_matmul(dtype, policy, left, right, out, rows, inner, columns, left_stride, right_stride,
                                  transpose_left, transpose_right, scratch, kStaticScratchBytes, status, stream);
}

// ============================================================================
// Row-sharded MatMul with the all-gather of C in the same kernel.  Every rank computes its rows
// of C with the full ordered K loop; the epilogue writes each finished tile into this device's
// C and, over NVLink, into every peer's C, so the all-gather overlaps the arithmetic tile by
// tile instead of following it.  The peers' buffers are mapped with CUDA IPC
// (pcu_b200_peer_alloc / pcu_b200_peer_open).  Plain stores only: no TMA or bulk copy ever
// reads or writes peer memory.
//
// Each buffer ends with a flag block (one word per rank): a CTA stores the call number into its
// own word of every peer's block when it starts, and waits, before its first store into a
// peer's C, until that peer's word in this rank's block has reached the call number.  A peer's
// kernel only starts once everything before it on the peer's stream has finished, so no store
// of this call can overwrite C while the peer is still reading the previous call's result.
// ============================================================================
namespace {

struct EntrySignal {
    unsigned long long *word[kMaxPeers];
    unsigned long long epoch;
    int count;
};

// The entry announcement of a call that has no tile to compute on this rank.
__global__ void announce_kernel(const __grid_constant__ EntrySignal sig) {
    if (threadIdx.x < (unsigned)sig.count)
        asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(sig.word[threadIdx.x]), "l"(sig.epoch) : "memory");
}

uint64_t peer_flags_offset(size_t elem, uint64_t rows_total, uint64_t columns) {
    return ((rows_total * columns * elem + 255) / 256) * 256;
}

}  // namespace

extern "C" size_t pcu_b200_peer_rows_bytes(int dtype, uint64_t rows_total, uint64_t columns) {
    if (dtype != PCU_B200_F32 && dtype != PCU_B200_F64) return 0;
    return peer_flags_offset(dtype == PCU_B200_F64 ? 8 : 4, rows_total, columns) + 256;
}

extern "C" int pcu_b200_strict_matmul_rows_allgather(int dtype, int policy, const void *left_rows, const void *right,
                                                     void *out_full, uint64_t row0, uint64_t rows,
                                                     uint64_t rows_total, uint64_t inner, uint64_t columns,
                                                     uint64_t left_stride, uint64_t right_stride, int transpose_right,
                                                     void *const *peer_outs, int npeers, int rank, uint64_t epoch,
                                                     void *workspace, size_t workspace_bytes, uint64_t *status,
                                                     void *stream) {
    if ((dtype != PCU_B200_F32 && dtype != PCU_B200_F64) || policy < 0 || policy > 2 || !status)
        return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (npeers < 0 || npeers > kMaxPeers || (npeers && !peer_outs)) return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (rank < 0 || rank > npeers || (npeers && epoch == 0)) return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (row0 > rows_total || rows > rows_total - row0) return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (!out_full) return PCU_B200_ERROR_INVALID_ARGUMENT;
    for (int q = 0; q < npeers; ++q)
        if (!peer_outs[q]) return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (rows > 0 && columns > 0 && inner > 0 && (!left_rows || !right)) return PCU_B200_ERROR_INVALID_ARGUMENT;
    const uint64_t right_row_len = transpose_right ? inner : columns;
    if (rows > 0 && columns > 0 && inner > 0 && (left_stride < inner || right_stride < right_row_len))
        return PCU_B200_ERROR_INVALID_ARGUMENT;
    unsigned __int128 events = (unsigned __int128)rows_total * columns;
    events *= (inner ? inner : 1);
    events *= 2;
    if (events > ((unsigned __int128)1 << 60)) return PCU_B200_ERROR_SIZE_OVERFLOW;
    const size_t elem = dtype == PCU_B200_F64 ? 8 : 4;
    const uint64_t flags = peer_flags_offset(elem, rows_total, columns);
    auto *st = reinterpret_cast<unsigned long long *>(status);
    cudaStream_t s = pcu_host::as_stream(stream);
    if (rows == 0 || columns == 0) {
        // No tile to store, but the call still counts on every rank: announce it so that peers
        // waiting on this rank's entry go on.
        if (!npeers) return PCU_B200_OK;
        EntrySignal sig{};
        sig.count = npeers;
        sig.epoch = epoch;
        for (int q = 0; q < npeers; ++q)
            sig.word[q] = reinterpret_cast<unsigned long long *>(static_cast<char *>(peer_outs[q]) + flags) + rank;
        announce_kernel<<<1, 32, 0, s>>>(sig);
        return pcu_host::launch_status();
    }
    const unsigned long long event_base = (unsigned long long)row0 * columns * (inner ? inner : 1) * 2;
    auto fill = [&](auto *typed_out) {
        using T = std::remove_pointer_t<decltype(typed_out)>;
        PeerSet<T> peers;
        peers.count = npeers;
        peers.epoch = epoch;
        for (int q = 0; q < npeers; ++q) {
            const int peer_rank = q < rank ? q : q + 1;
            char *peer = static_cast<char *>(peer_outs[q]);
            peers.out[q] = reinterpret_cast<T *>(peer + row0 * columns * elem);
            peers.signal[q] = reinterpret_cast<unsigned long long *>(peer + flags) + rank;
            peers.await_[q] = reinterpret_cast<const unsigned long long *>(static_cast<char *>(out_full) + flags) +
                              peer_rank;
        }
        return peers;
    };
    if (dtype == PCU_B200_F32) {
        const PeerSet<float> peers = fill(static_cast<float *>(nullptr));
        float *out = reinterpret_cast<float *>(static_cast<char *>(out_full) + row0 * columns * elem);
        return run_matmul<float>(policy, (const float *)left_rows, (const float *)right, out, rows, inner, columns,
                                 left_stride, right_stride, false, transpose_right != 0, workspace, workspace_bytes,
                                 st, s, ChainGuard{}, &peers, event_base);
    }
    const PeerSet<double> peers = fill(static_cast<double *>(nullptr));
    double *out = reinterpret_cast<double *>(static_cast<char *>(out_full) + row0 * columns * elem);
    return run_matmul<double>(policy, (const double *)left_rows, (const double *)right, out, rows, inner, columns,
                              left_stride, right_stride, false, transpose_right != 0, workspace, workspace_bytes, st,
                              s, ChainGuard{}, &peers, event_base);
}

extern "C" int pcu_b200_peer_alloc(size_t bytes, void **ptr, void *handle) {
    if (!ptr || !handle || !bytes) return PCU_B200_ERROR_INVALID_ARGUMENT;
    cudaError_t e = cudaMalloc(ptr, bytes);
    // zero-filled: the flag blocks of the row-sharded all-gather start below every call number
    if (e == cudaSuccess) e = cudaMemset(*ptr, 0, bytes);
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t *>(handle), *ptr);
    return e == cudaSuccess ? PCU_B200_OK : pcu_host::set_cuda_error(e);
}

extern "C" int pcu_b200_peer_open(const void *handle, void **ptr) {
    if (!ptr || !handle) return PCU_B200_ERROR_INVALID_ARGUMENT;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    return e == cudaSuccess ? PCU_B200_OK : pcu_host::set_cuda_error(e);
}

extern "C" int pcu_b200_peer_close(void *ptr) {
    const cudaError_t e = cudaIpcCloseMemHandle(ptr);
    return e == cudaSuccess ? PCU_B200_OK : pcu_host::set_cuda_error(e);
}

extern "C" int pcu_b200_peer_free(void *ptr) {
    const cudaError_t e = cudaFree(ptr);
    return e == cudaSuccess ? PCU_B200_OK : pcu_host::set_cuda_error(e);
}
