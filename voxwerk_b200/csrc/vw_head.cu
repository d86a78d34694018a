// vw_head.cu -- the vocabulary head GEMM on the 5th-generation tensor cores (tcgen05), ahead of the sampler.
//
// voxwerk computes each step's logits with TalkerModel.CodecHead (src/Voxwerk/Talker/TalkerModel.cs:133):
// logits[B, V] = hidden[B, H] x W^T, W = talker.codec_head.weight [V, H] (and CodePredictorHead, :136-137, for the
// 15 code-predictor heads).  Here hidden and W are bf16, the products accumulate in fp32 in tensor memory, and the
// fp32 logits go to a buffer the sampler reads right after (they are still in L2 for the sampler's pass).
//
// Kernel: one CTA per 128 x 256 output tile, 6 warps.
//   warp 0   TMA producer: K steps of 64 (A 128 x 64 and B 256 x 64 bf16 tiles, 128-byte swizzle) into a 4-stage
//            shared-memory ring, completing on mbarriers;
//   warp 1   allocates 256 TMEM columns; one elected thread issues tcgen05.mma (kind::f16, M 128, N 256, K 16) from
//            shared-memory descriptors, then tcgen05.commit frees each stage and finally signals the epilogue;
//   warps 2-5 epilogue: tcgen05.ld 32x32b (warp w reads TMEM lanes 32 (w % 4) ..), fp32 stores of the tile.
// Every mbarrier wait is bounded; on expiry the kernel sets an error bit, waits (bounded) for its own copies and
// MMAs, frees its TMEM and returns.  No cluster multicast anywhere.

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <atomic>
#include <mutex>

#include "vw_internal.h"

namespace vw {
namespace {

constexpr int kBM = 128, kBN = 256, kBK = 64, kStagesG = 4;
constexpr int kGemmThreads = 192;
constexpr uint32_t kStageBytesA = kBM * kBK * 2;    // 16 KB
constexpr uint32_t kStageBytesB = kBN * kBK * 2;    // 32 KB
constexpr uint64_t kGemmWaitNs = 2000000000ull;
constexpr uint32_t kTmemCols = 256;

struct __align__(1024) GemmSmem {
    uint8_t a[kStagesG][kStageBytesA];   // each stage 1024-byte aligned (128-byte swizzle atoms)
    uint8_t b[kStagesG][kStageBytesB];
    uint64_t full[kStagesG];
    uint64_t empty[kStagesG];
    uint64_t done;                       // all MMAs of the tile completed
    uint32_t tmem_base;
    int32_t abort;
};

__device__ __forceinline__ uint32_t s32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ bool try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(s32(bar)), "r"(parity), "r"(1000000u)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ bool wait_bounded(uint64_t* bar, uint32_t parity) {
    if (try_wait(bar, parity)) return true;
    const uint64_t t0 = now_ns();
    while (!try_wait(bar, parity))
        if (now_ns() - t0 > kGemmWaitNs) return false;
    return true;
}

// shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms 1024 bytes apart (SBO), version 1
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
    return static_cast<uint64_t>((saddr >> 4) & 0x3fffu) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
           (2ull << 61);
}
// instruction descriptor: fp32 accumulate, bf16 A and B, both K-major, N = 256, M = 128
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((kBN >> 3) << 17) | ((kBM >> 4) << 24);

__global__ void __launch_bounds__(kGemmThreads, 1)
head_gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b, int M, int N,
                 int K, float* __restrict__ out, int64_t ldo, unsigned* err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    GemmSmem& sm = *reinterpret_cast<GemmSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * kBN;
    const int nk = (K + kBK - 1) / kBK;   // a partial last step reads zeros past K (TMA fills out-of-range)

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStagesG; ++s) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(s32(&sm.full[s])));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(s32(&sm.empty[s])));
        }
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(s32(&sm.done)));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        sm.abort = 0;
    }
    if (warp == 1) {   // 256 TMEM columns for the 128 x 256 fp32 accumulator
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s32(&sm.tmem_base)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = sm.tmem_base;
    int issued = 0;       // producer: K steps whose copies were issued
    bool mma_done = false;

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer
        for (int k = 0; k < nk; ++k) {
            const int s = k % kStagesG;
            if (k >= kStagesG && !wait_bounded(&sm.empty[s], static_cast<uint32_t>(((k / kStagesG) - 1) & 1))) {
                atomicOr(err, kErrTimeout);
                sm.abort = 1;
                break;
            }
            if (*reinterpret_cast<volatile int32_t*>(&sm.abort)) break;
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(s32(&sm.full[s])),
                         "r"(kStageBytesA + kStageBytesB)
                         : "memory");
            asm volatile(
                "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                ::"r"(s32(sm.a[s])), "l"(reinterpret_cast<uint64_t>(&tma_a)), "r"(k * kBK), "r"(m0), "r"(s32(&sm.full[s]))
                : "memory");
            asm volatile(
                "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                ::"r"(s32(sm.b[s])), "l"(reinterpret_cast<uint64_t>(&tma_b)), "r"(k * kBK), "r"(n0), "r"(s32(&sm.full[s]))
                : "memory");
            issued = k + 1;
        }
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer (one thread)
        int k = 0;
        for (; k < nk; ++k) {
            const int s = k % kStagesG;
            if (!wait_bounded(&sm.full[s], static_cast<uint32_t>((k / kStagesG) & 1))) {
                atomicOr(err, kErrTimeout);
                sm.abort = 1;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t a0 = s32(sm.a[s]), b0 = s32(sm.b[s]);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk) {   // K 16 per instruction: 32 bytes further along the swizzled row
                const uint64_t da = umma_desc(a0 + 32 * kk), db = umma_desc(b0 + 32 * kk);
                const uint32_t acc = (k > 0 || kk > 0) ? 1u : 0u;
                asm volatile(
                    "{\n\t.reg .pred p;\n\t"
                    "setp.ne.b32 p, %4, 0;\n\t"
                    "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
                    ::"r"(tmem), "l"(da), "l"(db), "r"(kIdesc), "r"(acc)
                    : "memory");
            }
            // the stage is free once these MMAs have read it
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                s32(&sm.empty[s]))
                         : "memory");
        }
        // every MMA issued so far completes before `done` fires
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(s32(&sm.done))
                     : "memory");
        mma_done = k == nk;
    } else if (warp >= 2) {
        // ---------------- epilogue: TMEM -> registers -> fp32 logits
        const bool ok = wait_bounded(&sm.done, 0);
        if (!ok) {
            if (lane == 0) atomicOr(err, kErrTimeout);
        } else if (!*reinterpret_cast<volatile int32_t*>(&sm.abort)) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const int q = warp & 3;   // this warp's TMEM lane quarter
            const int row = m0 + 32 * q + lane;
            float* orow = out + static_cast<int64_t>(row) * ldo + n0;
#pragma unroll 1
            for (int c0 = 0; c0 < kBN; c0 += 32) {
                uint32_t v[32];
                const uint32_t addr = tmem + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(c0);
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
                    "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
                    : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                      "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
                      "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),
                      "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]),
                      "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
                    : "r"(addr));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (row < M) {
                    if (n0 + c0 + 32 <= N) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4)
                            *reinterpret_cast<float4*>(orow + c0 + j) =
                                make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]), __uint_as_float(v[j + 2]),
                                            __uint_as_float(v[j + 3]));
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (n0 + c0 + j < N) orow[c0 + j] = __uint_as_float(v[j]);
                    }
                }
            }
        }
    }
    // ---------------- teardown: own copies and MMAs finished, then TMEM freed
    if (warp == 0 && lane == 0) {
        for (int k = (issued > kStagesG ? issued - kStagesG : 0); k < issued; ++k)
            wait_bounded(&sm.full[k % kStagesG], static_cast<uint32_t>((k / kStagesG) & 1));
    }
    if (warp == 1 && lane == 0 && !mma_done) wait_bounded(&sm.done, 0);
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == 1) {
        __syncwarp();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
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

// bf16 [rows, K] row-major (row pitch `ld` elements) as 2-D tiles of box_rows x 64, 128-byte swizzle
bool make_map(CUtensorMap* m, const void* base, int rows, int K, int64_t ld, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

size_t head_gemm_smem_bytes() { return sizeof(GemmSmem) + 1024; }

cudaError_t launch_head_gemm(const void* a, int64_t lda, const void* b, int64_t ldb, int M, int N, int K, float* out,
                             int64_t ldo, unsigned* err, cudaStream_t stream) {
    if (M <= 0 || N <= 0) return cudaSuccess;
    CUtensorMap ma, mb;
    if (!make_map(&ma, a, M, K, lda, kBM) || !make_map(&mb, b, N, K, ldb, kBN)) return cudaErrorInvalidValue;
    const size_t smem = head_gemm_smem_bytes();
    static std::atomic<uint64_t> attr_set{0};   // one bit per device ordinal whose attribute is set
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_set.load(std::memory_order_acquire) & bit)) {
        e = cudaFuncSetAttribute(head_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        attr_set.fetch_or(bit, std::memory_order_acq_rel);
    }
    const dim3 grid((N + kBN - 1) / kBN, (M + kBM - 1) / kBM);
    head_gemm_kernel<<<grid, kGemmThreads, smem, stream>>>(ma, mb, M, N, K, out, ldo, err);
    return cudaGetLastError();
}

}  // namespace vw
