// vw_head.cu -- the vocabulary head GEMM on the 5th-generation tensor cores (tcgen05), ahead of the sampler.
//
// voxwerk computes each step's logits with TalkerModel.CodecHead (src/Voxwerk/Talker/TalkerModel.cs:133):
// logits[B, V] = hidden[B, H] x W^T, W = talker.codec_head.weight [V, H] (and CodePredictorHead, :136-137, for the
// 15 code-predictor heads).  Here hidden and W are bf16, the products accumulate in fp32 in tensor memory, and the
// fp32 logits go to a buffer the sampler reads right after (they are still in L2 for the sampler's pass).
//
// Kernel: persistent, one CTA per SM, output tiles of 128 x BN (BN chosen per shape on the host), 6 warps:
//   warp 0    TMA producer: K steps of 64 (A 128 x 64 and B BN x 64 bf16 boxes, 128-byte swizzle) into an S-stage
//             shared-memory ring, completing on mbarriers, running ahead across tile boundaries;
//   warp 1    owns the TMEM allocation (two BN-column fp32 accumulators); one elected thread issues tcgen05.mma
//             (kind::f16, M 128, N BN, K 16) from shared-memory descriptors; tcgen05.commit frees each stage and
//             hands a finished accumulator to the epilogue;
//   warps 2-5 epilogue: tcgen05.ld 32x32b (warp w owns TMEM lanes 32 (w % 4) ..), 32 x 32 fp32 blocks staged in
//             128-byte-swizzled shared memory and written by TMA stores (rows past M and columns past N are
//             clipped by the tensor map); the accumulator is released as soon as it is read, so the MMAs of the
//             next tile overlap this tile's stores.
// Every mbarrier wait is bounded; on expiry the kernel sets an error bit and every role stops; each role then waits
// (bounded) for its own copies and MMAs, the TMEM is freed and the kernel returns.  No cluster multicast anywhere.

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <mutex>

#include "vw_internal.h"

namespace vw {
namespace {

constexpr int kBM = 128, kBK = 64;
constexpr int kGemmThreads = 192;
constexpr uint32_t kStageBytesA = kBM * kBK * 2;   // 16 KB
constexpr uint32_t kEpiBuf = 32 * 32 * 4;          // one 32 x 32 fp32 block
constexpr uint32_t kRingBudget = 196608;           // bytes for the operand ring
constexpr uint64_t kGemmWaitNs = 2000000000ull;

constexpr uint32_t tmem_cols_for(int bn) {
    return 2 * bn <= 32 ? 32 : 2 * bn <= 64 ? 64 : 2 * bn <= 128 ? 128 : 2 * bn <= 256 ? 256 : 512;
}

template <int BN>
struct HeadCfg {
    static constexpr uint32_t kStageB = BN * kBK * 2;
    static constexpr uint32_t kStageBytes = kStageBytesA + kStageB;
    static constexpr int kStages = static_cast<int>(kRingBudget / kStageBytes < 12u ? kRingBudget / kStageBytes : 12u);
    static constexpr uint32_t kOffB = kStages * kStageBytesA;
    static constexpr uint32_t kOffEpi = kOffB + kStages * kStageB;   // 4 warps x 2 staging buffers
    static constexpr uint32_t kOffBar = kOffEpi + 8 * kEpiBuf;
    // full[S], empty[S], tmem_full[2], tmem_empty[2], done
    static constexpr uint32_t kOffMisc = kOffBar + (2 * kStages + 5) * 8;
    static constexpr uint32_t kBytes = kOffMisc + 16;
    static constexpr uint32_t kTmemCols = tmem_cols_for(BN);
    static constexpr uint32_t kAccStride = kTmemCols / 2;   // accumulator b starts at column b * kAccStride
    static_assert(kStages >= 2, "ring");
    static_assert(kBytes + 1024 <= 232448, "shared memory");
    static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "tile width");
    // instruction descriptor: fp32 accumulate, bf16 A and B, both K-major, N = BN, M = 128
    static constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((BN >> 3) << 17) | ((kBM >> 4) << 24);
};

__device__ __forceinline__ uint32_t s32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ bool try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(1000000u)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// true once the phase of `parity` completed; false on timeout (sets `err` and `abort`) or when another role aborted
__device__ bool wait_bounded(uint32_t bar, uint32_t parity, volatile int32_t* abort, unsigned* err) {
    if (try_wait(bar, parity)) return true;
    const uint64_t t0 = now_ns();
    while (!try_wait(bar, parity)) {
        if (*abort) return false;
        if (now_ns() - t0 > kGemmWaitNs) {
            atomicOr(err, kErrTimeout);
            *abort = 1;
            return false;
        }
    }
    return true;
}
// teardown flavour: bounded, no error reporting (an abort is already recorded)
__device__ void drain_wait(uint32_t bar, uint32_t parity) {
    const uint64_t t0 = now_ns();
    while (!try_wait(bar, parity))
        if (now_ns() - t0 > kGemmWaitNs) return;
}

// shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms 1024 bytes apart (SBO), version 1
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
    return static_cast<uint64_t>((saddr >> 4) & 0x3fffu) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
           (2ull << 61);
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

template <int BN>
__global__ void __launch_bounds__(kGemmThreads, 1)
head_gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                 const __grid_constant__ CUtensorMap tma_out, int M, int N, int K, unsigned* err) {
    using C = HeadCfg<BN>;
    constexpr int S = C::kStages;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = s32(sm);
    const uint32_t bar_full = sbase + C::kOffBar;   // + 8 s
    const uint32_t bar_empty = bar_full + 8 * S;    // + 8 s
    const uint32_t bar_tfull = bar_empty + 8 * S;   // + 8 b
    const uint32_t bar_tempty = bar_tfull + 16;     // + 8 b
    const uint32_t bar_done = bar_tempty + 16;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + C::kOffMisc);
    volatile int32_t* abort = reinterpret_cast<volatile int32_t*>(sm + C::kOffMisc + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_m = (M + kBM - 1) / kBM;
    const int tiles = tiles_m * ((N + BN - 1) / BN);
    const int nk = (K + kBK - 1) / kBK;   // a partial last step reads zeros past K (TMA fills out-of-range)

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar_full + 8 * s));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar_empty + 8 * s));
        }
        for (int b = 0; b < 2; ++b) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar_tfull + 8 * b));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 4;" ::"r"(bar_tempty + 8 * b));   // 4 epilogue warps
        }
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar_done));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        *abort = 0;
    }
    if (warp == 1) {   // two accumulators of BN fp32 columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s32(tmem_slot)),
                     "r"(C::kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer (one thread), running ahead across tiles
        if (lane == 0) {
            uint32_t it = 0;
            bool stop = false;
            for (int t = blockIdx.x; t < tiles && !stop; t += gridDim.x) {
                const int m0 = (t % tiles_m) * kBM, n0 = (t / tiles_m) * BN;
                for (int k = 0; k < nk; ++k, ++it) {
                    const uint32_t s = it % S;
                    if (it >= static_cast<uint32_t>(S) &&
                        !wait_bounded(bar_empty + 8 * s, ((it / S) - 1) & 1, abort, err)) {
                        stop = true;
                        break;
                    }
                    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar_full + 8 * s),
                                 "r"(C::kStageBytes)
                                 : "memory");
                    tma_load_2d(sbase + s * kStageBytesA, &tma_a, k * kBK, m0, bar_full + 8 * s);
                    tma_load_2d(sbase + C::kOffB + s * C::kStageB, &tma_b, k * kBK, n0, bar_full + 8 * s);
                }
            }
            // teardown: the copies still in flight land before the CTA may exit
            const uint32_t first = it > static_cast<uint32_t>(S) ? it - S : 0;
            for (uint32_t j = first; j < it; ++j) drain_wait(bar_full + 8 * (j % S), (j / S) & 1);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (one thread)
        if (lane == 0) {
            uint32_t it = 0, tc = 0;
            bool stop = false;
            for (int t = blockIdx.x; t < tiles && !stop; t += gridDim.x, ++tc) {
                const uint32_t buf = tc & 1;
                // the epilogue has read this accumulator's previous tile
                if (tc >= 2 && !wait_bounded(bar_tempty + 8 * buf, ((tc >> 1) - 1) & 1, abort, err)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t acc_addr = tmem + buf * C::kAccStride;
                for (int k = 0; k < nk; ++k, ++it) {
                    const uint32_t s = it % S;
                    if (!wait_bounded(bar_full + 8 * s, (it / S) & 1, abort, err)) {
                        stop = true;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t a0 = sbase + s * kStageBytesA, b0 = sbase + C::kOffB + s * C::kStageB;
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk) {   // K 16 per instruction: 32 bytes along the swizzled row
                        const uint64_t da = umma_desc(a0 + 32 * kk), db = umma_desc(b0 + 32 * kk);
                        const uint32_t accumulate = (k > 0 || kk > 0) ? 1u : 0u;
                        asm volatile(
                            "{\n\t.reg .pred p;\n\t"
                            "setp.ne.b32 p, %4, 0;\n\t"
                            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(acc_addr),
                            "l"(da), "l"(db), "r"(C::kIdesc), "r"(accumulate)
                            : "memory");
                    }
                    mma_commit(bar_empty + 8 * s);   // the stage is free once these MMAs have read it
                }
                if (stop) break;
                mma_commit(bar_tfull + 8 * buf);   // the accumulator is complete
            }
            // teardown: every MMA issued so far has completed before the TMEM is freed
            mma_commit(bar_done);
            drain_wait(bar_done, 0);
        }
    } else {
        // ---------------- epilogue: TMEM -> registers -> swizzled shared memory -> TMA store
        const int q = warp & 3;   // this warp's TMEM lane quarter: output rows 32 q .. 32 q + 31 of the tile
        const uint32_t epi = sbase + C::kOffEpi + q * 2 * kEpiBuf;
        uint32_t tc = 0, chunk = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++tc) {
            const int m0 = (t % tiles_m) * kBM, n0 = (t / tiles_m) * BN;
            const uint32_t buf = tc & 1;
            int ok = 1;
            if (lane == 0) ok = wait_bounded(bar_tfull + 8 * buf, (tc >> 1) & 1, abort, err) ? 1 : 0;
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const int row0 = m0 + 32 * q;
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32, ++chunk) {
                uint32_t v[32];
                const uint32_t addr = tmem + (static_cast<uint32_t>(32 * q) << 16) + buf * C::kAccStride + c0;
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
                    "%13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
                    "[%32];"
                    : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                      "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
                      "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),
                      "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]),
                      "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
                    : "r"(addr));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (c0 + 32 >= BN) {   // last read of this accumulator: hand it back to the MMA issuer
                    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                    __syncwarp();
                    if (lane == 0)
                        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar_tempty + 8 * buf) : "memory");
                }
                if (row0 >= M || n0 + c0 >= N) continue;   // no part of this block lies inside the output
                const uint32_t sb = epi + (chunk & 1) * kEpiBuf;
                // the TMA store that last read this staging buffer has finished reading it
                if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
                __syncwarp();
                // row `lane`, 16-byte piece j of 8 at position j ^ (lane & 7): the 128-byte swizzle of the store map
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint32_t dst = sb + lane * 128 + ((j ^ (lane & 7)) << 4);
                    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(v[4 * j]),
                                 "r"(v[4 * j + 1]), "r"(v[4 * j + 2]), "r"(v[4 * j + 3])
                                 : "memory");
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // visible to the TMA engine
                __syncwarp();
                if (lane == 0) {
                    asm volatile(
                        "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                            reinterpret_cast<uint64_t>(&tma_out)),
                        "r"(n0 + c0), "r"(row0), "r"(sb)
                        : "memory");
                    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                }
            }
        }
        // teardown: this warp's stores have completed before its shared memory goes away
        if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        __syncwarp();
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == 1) {
        __syncwarp();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::kTmemCols));
    }
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda)
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn() {
    static std::once_flag once;
    static EncodeTiledFn fn = nullptr;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// row-major [rows, cols] (row pitch `ld` elements of `esize` bytes) in boxes of box_rows x box_cols (128 bytes wide),
// 128-byte swizzle
bool make_map(CUtensorMap* m, CUtensorMapDataType type, size_t esize, const void* base, int rows, int cols, int64_t ld,
              int box_rows, int box_cols) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * esize};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, type, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count_of(int dev) {
    static std::atomic<int> cache[64];
    std::atomic<int>& c = cache[dev & 63];
    int n = c.load(std::memory_order_relaxed);
    if (n <= 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        c.store(n, std::memory_order_relaxed);
    }
    return n;
}

template <int BN>
cudaError_t launch_bn(const CUtensorMap& ma, const void* b, int64_t ldb, const CUtensorMap& mo, int M, int N, int K,
                      unsigned* err, int dev, int sms, cudaStream_t stream) {
    using C = HeadCfg<BN>;
    CUtensorMap mb;
    if (!make_map(&mb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, b, N, K, ldb, BN, kBK)) return cudaErrorInvalidValue;
    static std::atomic<uint64_t> attr_set{0};   // one bit per device ordinal whose attribute is set
    const uint64_t bit = 1ull << (dev & 63);
    const size_t smem = C::kBytes + 1024;
    if (!(attr_set.load(std::memory_order_acquire) & bit)) {
        cudaError_t e = cudaFuncSetAttribute(head_gemm_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        attr_set.fetch_or(bit, std::memory_order_acq_rel);
    }
    const int tiles = ((M + kBM - 1) / kBM) * ((N + BN - 1) / BN);
    head_gemm_kernel<BN><<<std::min(tiles, sms), kGemmThreads, smem, stream>>>(ma, mb, mo, M, N, K, err);
    return cudaGetLastError();
}

}  // namespace

// The tile width whose persistent schedule finishes first: waves x cost of one 64-deep K step, the larger of the
// MMA (128 x BN x 64 at 8192 flop per cycle: 2 BN cycles) and the operand fill (16 KB + 128 BN bytes at about
// 128 bytes per cycle).  Ties go to the wider tile (fewer re-reads of the hidden rows).
int head_gemm_tile_n(int M, int N, int sms) {
    static const int kWidths[] = {256, 192, 128, 96, 64, 32};
    int best = 256;
    int64_t best_cost = -1;
    for (int bn : kWidths) {
        const int64_t tiles = static_cast<int64_t>((M + kBM - 1) / kBM) * ((N + bn - 1) / bn);
        const int64_t waves = (tiles + sms - 1) / sms;
        const int64_t cost = waves * std::max<int64_t>(2 * bn, 128 + bn);
        if (best_cost < 0 || cost < best_cost) {
            best = bn;
            best_cost = cost;
        }
    }
    return best;
}

cudaError_t launch_head_gemm(const void* a, int64_t lda, const void* b, int64_t ldb, int M, int N, int K, float* out,
                             int64_t ldo, unsigned* err, cudaStream_t stream) {
    if (M <= 0 || N <= 0) return cudaSuccess;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const int sms = sm_count_of(dev);
    CUtensorMap ma, mo;
    if (!make_map(&ma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a, M, K, lda, kBM, kBK) ||
        !make_map(&mo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, out, M, N, ldo, 32, 32))
        return cudaErrorInvalidValue;
    switch (head_gemm_tile_n(M, N, sms)) {
        case 256: return launch_bn<256>(ma, b, ldb, mo, M, N, K, err, dev, sms, stream);
        case 192: return launch_bn<192>(ma, b, ldb, mo, M, N, K, err, dev, sms, stream);
        case 128: return launch_bn<128>(ma, b, ldb, mo, M, N, K, err, dev, sms, stream);
        case 96: return launch_bn<96>(ma, b, ldb, mo, M, N, K, err, dev, sms, stream);
        case 64: return launch_bn<64>(ma, b, ldb, mo, M, N, K, err, dev, sms, stream);
        default: return launch_bn<32>(ma, b, ldb, mo, M, N, K, err, dev, sms, stream);
    }
}

}  // namespace vw
