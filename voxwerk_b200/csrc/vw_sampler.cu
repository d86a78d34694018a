// vw_sampler.cu -- fused token-sampling kernels for sm_100a (B200).
//
// Two kernels per call, stream-ordered:
//   * row_warp_kernel (vw_rowwarp.cuh): one warp per row, every row of the call.  It finishes greedy rows and
//     sampling rows with 0 < top-k <= 64 from a candidate set, reading each row once with 16-byte loads, and
//     appends every other row to a deferred list.
//   * whole_row_kernel: the deferred rows (top-k off or > 64, a penalty < 1, unaligned rows, candidate overflow),
//     CTAs of five warps: a producer warp streams each row's logits and history into a shared-memory ring with
//     cp.async.bulk (TMA bulk copies) completing on mbarriers, and four element warps hold the row in registers.
//     The suppressed span of talker rows is never read by either kernel.
//
// Per row, in the order of the reference (src/Voxwerk/Talker/Sampler.cs, TalkerGenerator.cs):
//   1. repetition penalty (talker rows; Sampler.cs:25-33): history ids -> a flag byte per id (Distinct());
//      each element whose bit is set becomes s < 0 ? s * p : s / p in fp32.  The IEEE quotient s / p is formed
//      as fp32(fp64(s) * RN64(1/p)): the fp64 product is within 2^-52 relative of s/p while no fp32 rounding
//      midpoint lies closer than 2^-49 relative to a quotient of two fp32 values, so both round the same way.
//      The warp kernel applies a penalty > 1 to the candidates only (it only lowers values, so the unpenalized
//      value decides first whether an element can be a candidate at all).
//   2. suppress mask (talker rows; TalkerGenerator.cs:247-248): ids [lo, hi) except EOS, and EOS while
//      t < min_new_tokens, become -inf.
//   3. greedy rows: first index of the maximum (Sampler.cs:90-95).
//   4. temperature: x * fp32(1/T) (Sampler.cs:39-40).
//   5. top-k (Sampler.cs:42-49): every value >= the K-th largest survives (ties kept).  For K <= 64 the
//      candidates are the values >= tau for a threshold tau with K <= count <= 128, so the K-th largest is
//      >= tau: tau is carried from the warp's previous row of the same segment and options (and from call to
//      call), or else rebuilt from the row (the K-th largest of the lanes' top-2 values).  Otherwise a binned
//      select over the row finds the K-th largest.
//   6. softmax in fp64, top-p cut over the (prob, index)-ascending order and the inverse-CDF draw
//      (Sampler.cs:51-88).  The reference's sums are sequential fp64 roundings.  Here they are formed in
//      parallel; every decision they feed (which ids top-p removes, where the draw lands) is taken only when the
//      parallel value is farther from the threshold than a proven bound on the difference between the two
//      (eta = (6n + 128) 2^-53 of the total for n survivors on the candidate path, (8n + 128) 2^-53 where
//      fixed-point histograms are involved, covering the reference's n-term sequential roundings and this
//      code's own roundings, with room for a 1-ulp exp difference although the device exp is the host libm's).  A row with any decision inside that band is
//      replayed in the reference's exact sequential order (replay paths below), so the ids equal the
//      reference's in every case.
//
// Compile with -fmad=false: no multiply-add may be contracted; every rounding step is explicit (_rn
// intrinsics) to match the reference's separately rounded fp32 / fp64 operations.

#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <mutex>
#include <cuda_runtime.h>

#include "vw_libm_exp.h"
#include "vw_internal.h"

namespace vw {
namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr double kU = 1.1102230246251565e-16;      // 2^-53
constexpr double kFix = 1099511627776.0;            // 2^40: fixed-point scale of histogram masses (e <= 1): two
                                                    // 20-bit parts, each bin's sum of 3072 parts fits 32 bits
constexpr int kProducerWarp = kWarps;              // warp 4
constexpr int kBlockThreads = (kWarps + 1) * 32;   // 160

// Everything the element warps need about a row, prepared by the producer warp.  Kept in its own ring of 2 x
// n_stages entries, so an entry outlives the early release of its row's stage.
struct __align__(16) RowMeta {
    double uniform;               // the row's NextDouble() draw
    double pen_rcp;               // RN64(1 / repetition penalty)
    const unsigned char* row_ptr; // the row in global memory (unaligned rows are staged by the element warps)
    const int32_t* hist;          // the row's history ids in global memory
    int32_t* out_id;              // where the row's id goes
    double* out_probs;            // the row's probability output, or null
    int32_t row, seg, opt_idx, step;
    int32_t hist_len, hs_lo, hs_hi;   // history ids [hs_lo, hs_hi) are staged in shared memory
    int32_t lo_al, hi_al;         // staged logits: ids [0, lo_al) | kvw ids from kbase (the EOS vector) | [hi_al, V)
    int32_t kvw, kbase;
    int32_t direct;               // logits were not bulk-copied: the element warps load them
    int32_t pen_on;               // repetition penalty active
    int32_t opt_ok;               // option index valid
    int32_t V, dtype, kind;
    int32_t sup_lo, sup_hi, eos, eos_blocked;
    int32_t slow_vlo, slow_vhi, eos_vec;   // staged vectors that need the per-element mask rules
    float inv_t;                  // fp32(1 / T)
    DevOptions opt;
};
static_assert(sizeof(RowMeta) % 16 == 0, "RowMeta alignment");

struct Cand {
    float x;
    int32_t idx;
};


// Binned-search histograms: counts and the three 20-bit chunks of fixed-point masses per bin.
struct Bins {
    uint32_t cnt[256];
    uint32_t m[3][256];
};

struct __align__(16) SmemMisc {
    float tau_w[kWarps];
    float red_f[8][kWarps];
    int32_t red_i[8][kWarps];
    double red_d[8][kWarps];
    unsigned long long red_u[4][kWarps];
    double red_v[kWarps][8];
    int32_t issued;       // rows the producer has issued (timeout drain)
    uint32_t progress;    // rows finished by the element warps (extends the producer's wait bound)
    uint32_t cand_count[2];   // candidate counters, alternating by row (reset one row after use)
    int32_t bc_i[4];
    unsigned long long bc_u[2];
    double bc_d[4];
    union __align__(16) {
        Bins bins;        // whole-row path histograms
    } u;
    int32_t flags[kCandCap];   // candidate replay scratch
};

// ---------------------------------------------------------------- PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
// Waits for the phase with `parity` to complete; the thread sleeps in the barrier for up to kSuspendNs per try
// instead of spinning (a spinning warp would take issue slots from the working warps of its SM).
constexpr uint32_t kSuspendNs = 1000000;   // 1 ms per try; the phase completing wakes the thread at once
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendNs)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Gives up after `limit_ns` without progress and returns false.  `progress` (nullable) is a counter whose change
// restarts the clock.
__device__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint64_t limit_ns,
                                  const volatile uint32_t* progress = nullptr) {
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t0 = global_ns();
    uint32_t last = progress ? *progress : 0u;
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (progress) {
            const uint32_t now = *progress;
            if (now != last) {
                last = now;
                t0 = global_ns();
            }
        }
        if (global_ns() - t0 > limit_ns) return false;
    }
}
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// TMA bulk copy global -> shared, completing `bytes` on `bar`.  dst, src 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// Barrier among the 128 element threads (named barrier 1; the producer warp never joins it).
__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
__device__ __forceinline__ bool cbar_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, 1, 128, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(v))
        : "memory");
    return r != 0;
}

// ---------------------------------------------------------------- value helpers
// Position k of the stage ring, kept incrementally (no integer division per row): stage s = k % S, round
// n = k / S; the meta slot k % (2 S) is s + S (n & 1).
struct RingPos {
    int s, n;
    __device__ __forceinline__ void next(int S) {
        if (++s == S) {
            s = 0;
            ++n;
        }
    }
    __device__ __forceinline__ int meta(int S) const { return s + (n & 1) * S; }
};

__device__ __forceinline__ float neg_inf() { return __int_as_float(0xff800000); }
__device__ __forceinline__ float pos_inf() { return __int_as_float(0x7f800000); }
__device__ __forceinline__ bool is_neg_inf(float x) { return __float_as_uint(x) == 0xff800000u; }

// Order-preserving uint32 key of a float; -0 is folded onto +0 (they compare equal in every rule here).
__device__ __forceinline__ uint32_t okey(float x) {
    uint32_t u = __float_as_uint(x);
    if ((u & 0x7fffffffu) == 0) u = 0;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float okey_inv(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}
// exp(fp64(fp32(x - mx))), Sampler.cs:57, with the host libm's exact exp (vw_libm_exp.h): the replays then
// reproduce the reference's sums bit for bit, and the parallel paths' bands need no allowance for exp.
__device__ __forceinline__ double softmax_num(float x, float mx) {
    return libm_exp(static_cast<double>(__fsub_rn(x, mx)));
}

__device__ __forceinline__ uint64_t shfl_xor_u64(uint64_t v, int m) { return __shfl_xor_sync(kFull, v, m); }
__device__ __forceinline__ uint64_t shfl_u64(uint64_t v, int src) { return __shfl_sync(kFull, v, src); }
__device__ __forceinline__ double shfl_d(double v, int src) { return __shfl_sync(kFull, v, src); }

// Bitonic sort of 32*P uint64 keys held slot-major (element e = slot * 32 + lane), ascending.
template <int P>
__device__ __forceinline__ void warp_sort(uint64_t (&k)[P], int lane) {
#pragma unroll
    for (int size = 2; size <= 32 * P; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            if (stride >= 32) {
                const int ds = stride >> 5;
#pragma unroll
                for (int s = 0; s < P; ++s) {
                    const int t = s ^ ds;
                    if (t > s) {
                        const bool up = (((s * 32 + lane) & size) == 0);
                        const uint64_t a = k[s], b = k[t];
                        const bool sw = up ? (a > b) : (a < b);
                        k[s] = sw ? b : a;
                        k[t] = sw ? a : b;
                    }
                }
            } else {
#pragma unroll
                for (int s = 0; s < P; ++s) {
                    const uint64_t o = shfl_xor_u64(k[s], stride);
                    const bool lower = (lane & stride) == 0;
                    const bool up = (((s * 32 + lane) & size) == 0);
                    const uint64_t mn = k[s] < o ? k[s] : o;
                    const uint64_t mx = k[s] < o ? o : k[s];
                    k[s] = (lower == up) ? mn : mx;
                }
            }
        }
    }
}

// Bitonic sort of 32*P uint32 keys held slot-major, ascending.
template <int P>
__device__ __forceinline__ void warp_sort32(uint32_t (&k)[P], int lane) {
#pragma unroll
    for (int size = 2; size <= 32 * P; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            if (stride >= 32) {
                const int ds = stride >> 5;
#pragma unroll
                for (int s = 0; s < P; ++s) {
                    const int t = s ^ ds;
                    if (t > s) {
                        const bool up = (((s * 32 + lane) & size) == 0);
                        const uint32_t a = k[s], b = k[t];
                        k[s] = up ? min(a, b) : max(a, b);
                        k[t] = up ? max(a, b) : min(a, b);
                    }
                }
            } else {
#pragma unroll
                for (int s = 0; s < P; ++s) {
                    const uint32_t o = __shfl_xor_sync(kFull, k[s], stride);
                    const bool lower = (lane & stride) == 0;
                    const bool up = (((s * 32 + lane) & size) == 0);
                    k[s] = (lower == up) ? min(k[s], o) : max(k[s], o);
                }
            }
        }
    }
}

// Same network on (key, tag) pairs ordered lexicographically; tags are unique so the order is total.
template <int P>
__device__ __forceinline__ void warp_sort_pair(uint64_t (&k)[P], uint32_t (&t)[P], int lane) {
#pragma unroll
    for (int size = 2; size <= 32 * P; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            if (stride >= 32) {
                const int ds = stride >> 5;
#pragma unroll
                for (int s = 0; s < P; ++s) {
                    const int u = s ^ ds;
                    if (u > s) {
                        const bool up = (((s * 32 + lane) & size) == 0);
                        const bool a_lt_b = k[s] < k[u] || (k[s] == k[u] && t[s] < t[u]);
                        const bool sw = up ? !a_lt_b : a_lt_b;
                        const uint64_t ka = k[s], kb = k[u];
                        const uint32_t ta = t[s], tb = t[u];
                        k[s] = sw ? kb : ka;
                        k[u] = sw ? ka : kb;
                        t[s] = sw ? tb : ta;
                        t[u] = sw ? ta : tb;
                    }
                }
            } else {
#pragma unroll
                for (int s = 0; s < P; ++s) {
                    const uint64_t ko = shfl_xor_u64(k[s], stride);
                    const uint32_t to = __shfl_xor_sync(kFull, t[s], stride);
                    const bool lower = (lane & stride) == 0;
                    const bool up = (((s * 32 + lane) & size) == 0);
                    const bool me_lt = k[s] < ko || (k[s] == ko && t[s] < to);
                    const bool take_mine = (lower == up) ? me_lt : !me_lt;
                    k[s] = take_mine ? k[s] : ko;
                    t[s] = take_mine ? t[s] : to;
                }
            }
        }
    }
}

// Warp reductions; results are the same in every lane (lane 0's value is broadcast where rounding is involved).
__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
    return v;
}
__device__ __forceinline__ float warp_min_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(kFull, v, o));
    return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}
__device__ __forceinline__ int warp_max_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(kFull, v, o));
    return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __dadd_rn(v, __shfl_xor_sync(kFull, v, o));
    return __shfl_sync(kFull, v, 0);
}
// Inclusive / exclusive prefix sums across the 32 lanes.
__device__ __forceinline__ double warp_incl_d(double v, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double y = __shfl_up_sync(kFull, v, o);
        if (lane >= o) v = __dadd_rn(v, y);
    }
    return v;
}
__device__ __forceinline__ double warp_excl_from_incl_d(double incl, int lane) {
    const double y = __shfl_up_sync(kFull, incl, 1);
    return lane == 0 ? 0.0 : y;
}

// ---------------------------------------------------------------- block reductions (128 element threads)
// Each call site passes its own `slot`; a slot is reused only after at least one more cbar.
__device__ __forceinline__ float block_max_f(float v, SmemMisc& m, int slot, int lane, int warp) {
    v = warp_max_f(v);
    if (lane == 0) m.red_f[slot][warp] = v;
    cbar();
    float r = m.red_f[slot][0];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) r = fmaxf(r, m.red_f[slot][w]);
    return r;
}
__device__ __forceinline__ int block_sum_i(int v, SmemMisc& m, int slot, int lane, int warp) {
    v = warp_sum_i(v);
    if (lane == 0) m.red_i[slot][warp] = v;
    cbar();
    int r = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) r += m.red_i[slot][w];
    return r;
}
__device__ __forceinline__ int block_max_i(int v, SmemMisc& m, int slot, int lane, int warp) {
    v = warp_max_i(v);
    if (lane == 0) m.red_i[slot][warp] = v;
    cbar();
    int r = m.red_i[slot][0];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) r = max(r, m.red_i[slot][w]);
    return r;
}
__device__ __forceinline__ double block_sum_d(double v, SmemMisc& m, int slot, int lane, int warp) {
    v = warp_sum_d(v);
    if (lane == 0) m.red_d[slot][warp] = v;
    cbar();
    double r = m.red_d[slot][0];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) r = __dadd_rn(r, m.red_d[slot][w]);
    return r;
}
// max of a and min of b in one barrier (slots `slot` of red_f for a and `slot + 1` for b)
__device__ __forceinline__ void block_max_min_f(float& a, float& b, SmemMisc& m, int slot, int lane, int warp) {
    a = warp_max_f(a);
    b = warp_min_f(b);
    if (lane == 0) {
        m.red_f[slot][warp] = a;
        m.red_f[slot + 1][warp] = b;
    }
    cbar();
    a = m.red_f[slot][0];
    b = m.red_f[slot + 1][0];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) {
        a = fmaxf(a, m.red_f[slot][w]);
        b = fminf(b, m.red_f[slot + 1][w]);
    }
}
// Exclusive scan of a uint64 over the 128 element threads in thread order; `total` is the sum over all.
__device__ __forceinline__ void block_scan_u64(unsigned long long v, SmemMisc& m, int slot, int lane, int warp,
                                               unsigned long long& excl, unsigned long long& total) {
    unsigned long long incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long y = __shfl_up_sync(kFull, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) m.red_u[slot][warp] = incl;
    cbar();
    unsigned long long base = 0, tot = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
        const unsigned long long t = m.red_u[slot][w];
        if (w < warp) base += t;
        tot += t;
    }
    excl = base + incl - v;
    total = tot;
}

// ---------------------------------------------------------------- per-row element transform
struct RowCtx {
    int vocab;
    int kind;            // 0 talker
    int sup_lo, sup_hi, eos;
    bool eos_blocked;    // t < min_new_tokens
    bool pen_on;
    float pen;
    double pen_rcp;      // RN64(1 / pen)
    bool sample;
    float inv_t;         // fp32(1 / T)
    const uint8_t* flags;     // flags[id] = 1: id is in the history (Distinct()); penalised when pen_on
    int slow_vlo, slow_vhi;   // staged vectors that may hold suppressed ids
    int eos_vec;              // staged vector holding a suppressed EOS, or -1
};

// Staged position -> vocabulary id: [0, lo_al) | kvw ids from kbase | [hi_al, V)
struct RowMap {
    int lo_al, kvw, kbase, hi_al;
    __device__ __forceinline__ int idx(int q) const {
        if (q < lo_al) return q;
        q -= lo_al;
        if (q < kvw) return kbase + q;
        return q - kvw + hi_al;
    }
    // vocabulary id -> staged position, or -1 for an id inside the unstaged (suppressed) span
    __device__ __forceinline__ int pos(int id) const {
        if (id < lo_al) return id;
        if (id >= kbase && id < kbase + kvw) return lo_al + (id - kbase);
        if (id >= hi_al) return lo_al + kvw + (id - hi_al);
        return -1;
    }
};

// Sampler.cs:31 in fp32: s < 0 ? s * p : s / p, the quotient as fp32(fp64(s) * RN64(1/p)) (see the file header).
__device__ __forceinline__ float penalize(float s, float pen, double pen_rcp) {
    return s < 0.0f ? __fmul_rn(s, pen) : __double2float_rn(__dmul_rn(static_cast<double>(s), pen_rcp));
}

// penalty (Sampler.cs:31) -> mask (TalkerGenerator.cs:247-248) -> temperature (Sampler.cs:40); `pen`: the id is
// in the history
__device__ __forceinline__ float transform(float v, int idx, bool pen, const RowCtx& c) {
    if (c.pen_on && pen) v = penalize(v, c.pen, c.pen_rcp);
    if (c.kind == 0) {
        const bool masked = (idx >= c.sup_lo && idx < c.sup_hi && idx != c.eos) || (idx == c.eos && c.eos_blocked);
        if (masked) v = neg_inf();
    }
    if (c.sample) v = __fmul_rn(v, c.inv_t);
    return v;
}

// Bit e set: id i0 + e is in the history (its flag byte is 1).  i0 is a multiple of VW.
template <int VW>
__device__ __forceinline__ uint32_t pen_mask(const uint8_t* flags, int i0) {
    uint32_t m = 0u;
#pragma unroll
    for (int w = 0; w < VW / 4; ++w) {
        const uint32_t f = reinterpret_cast<const uint32_t*>(flags + i0)[w];   // four 0/1 bytes
        m |= ((f & 1u) | ((f >> 7) & 2u) | ((f >> 14) & 4u) | ((f >> 21) & 8u)) << (4 * w);
    }
    return m;
}

template <int VW>
__device__ __forceinline__ void load_vec(const unsigned char* base, int qv, float (&v)[VW]);

template <>
__device__ __forceinline__ void load_vec<4>(const unsigned char* base, int qv, float (&v)[4]) {
    const float4 f = reinterpret_cast<const float4*>(base)[qv];
    v[0] = f.x;
    v[1] = f.y;
    v[2] = f.z;
    v[3] = f.w;
}
template <>
__device__ __forceinline__ void load_vec<8>(const unsigned char* base, int qv, float (&v)[8]) {
    const uint4 u = reinterpret_cast<const uint4*>(base)[qv];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        v[2 * j] = __uint_as_float(w[j] << 16);             // Bf16.ToFloat (Bf16.cs:13)
        v[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
    }
}

__device__ __forceinline__ float load_elem(const unsigned char* base, int i, int dtype) {
    if (dtype == 0) return reinterpret_cast<const float*>(base)[i];
    return __uint_as_float(static_cast<uint32_t>(reinterpret_cast<const uint16_t*>(base)[i]) << 16);
}

// ---------------------------------------------------------------- exact block path (all 128 element threads)
// The reference's operations in its own order over gx[0, V) (per-CTA global scratch; suppressed ids = -inf).
// Runs for rows whose parallel decisions are inside the error band, and for rows of more than 3072 active ids.
__device__ int exact_block_path(const RowCtx& c, const DevOptions& o, double r, float mx, float* gx, double* gp,
                                uint4* gs, int sort_n, double* out_probs, SmemMisc& misc, int tid) {
    const int V = c.vocab;
    if (is_neg_inf(mx)) {
        // Every logit is -inf: the reference's probabilities are 0/0 = NaN, the draw never fires and it
        // returns the last index (Sampler.cs:80-87).
        if (out_probs)
            for (int i = tid; i < V; i += kThreads) out_probs[i] = 0.0;
        cbar();
        return V - 1;
    }
    float kth = neg_inf();
    const int K = o.top_k;
    if (K > 0 && K < V) {   // the K-th largest of the V values
        uint32_t prefix = 0, pmask = 0;
        int need = K;
        for (int shift = 24; shift >= 0; shift -= 8) {
            for (int b = tid; b < 256; b += kThreads) misc.u.bins.cnt[b] = 0;
            cbar();
            for (int i = tid; i < V; i += kThreads) {
                const uint32_t k = okey(gx[i]);
                if ((k & pmask) == prefix) atomicAdd(&misc.u.bins.cnt[(k >> shift) & 255u], 1u);
            }
            cbar();
            if (tid == 0) {
                int d = 255;
                for (; d > 0; --d) {
                    const int h = static_cast<int>(misc.u.bins.cnt[d]);
                    if (need <= h) break;
                    need -= h;
                }
                misc.bc_i[0] = d;
                misc.bc_i[1] = need;
            }
            cbar();
            const uint32_t d = static_cast<uint32_t>(misc.bc_i[0]);
            need = misc.bc_i[1];
            prefix |= d << shift;
            pmask |= 255u << shift;
            cbar();
        }
        kth = okey_inv(prefix);
    }
    for (int i = tid; i < V; i += kThreads) {   // Sampler.cs:55-57
        const float x = gx[i];
        gp[i] = (!is_neg_inf(x) && x >= kth) ? softmax_num(x, mx) : 0.0;
    }
    cbar();
    if (tid == 0) {   // sequential fp64 sum in index order (Sampler.cs:58)
        double s = 0.0;
        for (int i = 0; i < V; ++i) {
            const double v = gp[i];
            if (v != 0.0) s = __dadd_rn(s, v);
        }
        misc.bc_d[0] = s;
    }
    cbar();
    {
        const double s1 = misc.bc_d[0];
        for (int i = tid; i < V; i += kThreads) gp[i] = __ddiv_rn(gp[i], s1);   // :60
    }
    cbar();
    if (o.top_p < 1.0f) {   // Sampler.cs:62-75
        const double thr = static_cast<double>(__fsub_rn(1.0f, o.top_p));
        for (int i = tid; i < sort_n; i += kThreads) {
            uint4 it;
            if (i < V) {
                const unsigned long long b = static_cast<unsigned long long>(__double_as_longlong(gp[i]));
                it = make_uint4(static_cast<uint32_t>(b), static_cast<uint32_t>(b >> 32), static_cast<uint32_t>(i),
                                0u);
            } else {
                it = make_uint4(0xffffffffu, 0xffffffffu, 0xffffffffu, 0u);
            }
            gs[i] = it;
        }
        cbar();
        // Bitonic sort by (prob, index) ascending == stable OrderBy(prob) (Sampler.cs:65).
        for (int size = 2; size <= sort_n; size <<= 1) {
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                for (int i = tid; i < sort_n / 2; i += kThreads) {
                    const int lo = 2 * stride * (i / stride) + (i % stride);
                    const int hi = lo + stride;
                    const bool up = (lo & size) == 0;
                    const uint4 a = gs[lo], b = gs[hi];
                    const uint64_t ka = (static_cast<uint64_t>(a.y) << 32) | a.x;
                    const uint64_t kb = (static_cast<uint64_t>(b.y) << 32) | b.x;
                    const bool a_lt_b = ka < kb || (ka == kb && a.z < b.z);
                    if (up ? !a_lt_b : a_lt_b) {
                        gs[lo] = b;
                        gs[hi] = a;
                    }
                }
                cbar();
            }
        }
        if (tid == 0) {   // cumulative cut over the ascending order, never the last element (:67-72)
            double cum = 0.0;
            int m = V - 1;
            for (int j = 0; j < V - 1; ++j) {
                const uint4 it = gs[j];
                const double v =
                    __longlong_as_double(static_cast<long long>((static_cast<uint64_t>(it.y) << 32) | it.x));
                if (v == 0.0) continue;   // adds 0 and removes an id that is already 0
                cum = __dadd_rn(cum, v);
                if (!(cum <= thr)) {
                    m = j;
                    break;
                }
            }
            misc.bc_i[0] = m;
        }
        cbar();
        {
            const int m = misc.bc_i[0];
            for (int j = tid; j < m; j += kThreads) gp[gs[j].z] = 0.0;
        }
        cbar();
        if (tid == 0) {   // probs.Sum() in index order (:73)
            double s = 0.0;
            for (int i = 0; i < V; ++i) {
                const double v = gp[i];
                if (v != 0.0) s = __dadd_rn(s, v);
            }
            misc.bc_d[0] = s;
        }
        cbar();
        {
            const double s2 = misc.bc_d[0];
            for (int i = tid; i < V; i += kThreads) gp[i] = __ddiv_rn(gp[i], s2);   // :74
        }
        cbar();
    }
    if (tid == 0) {   // inverse-CDF draw (Sampler.cs:77-87)
        double acc = 0.0;
        int last = 0, res = -1;
        for (int i = 0; i < V; ++i) {
            const double v = gp[i];
            if (v <= 0.0) continue;
            acc = __dadd_rn(acc, v);
            last = i;
            if (r < acc) {
                res = i;
                break;
            }
        }
        misc.bc_i[0] = res < 0 ? last : res;
    }
    if (out_probs)
        for (int i = tid; i < V; i += kThreads) out_probs[i] = gp[i];
    cbar();
    const int res = misc.bc_i[0];
    cbar();
    return res;
}

// ---------------------------------------------------------------- binned search (element threads)
// Ascending search over the values x[j] whose bit j is set in `live`: finds the value v* at which the running
// weight, from the smallest value up, first exceeds `target` (weights: counts, or fixed-point masses
// round(ev(j) * 2^40) when kMass, binned without counts: two shared atomics per value).  On return `below` is the
// weight of the live values < v* and `cnt` the number of live values equal to v*.  Each pass bins the live values linearly over [min, max] (monotone in the value),
// keeps the bin holding the crossing, and stops when one value is left.  Returns false (the caller replays the
// row) when the span is not a finite positive float or eight passes do not isolate a value.
template <bool kMass, typename EvFn>
__device__ bool binned_search(const float (&x)[kRegElems], uint32_t live, EvFn ev, unsigned long long target,
                              SmemMisc& m, int tid, int lane, int warp, float& vstar, unsigned long long& below,
                              int& cnt) {
    float lo = pos_inf(), hi = neg_inf();
    int n = 0;
#pragma unroll
    for (int j = 0; j < kRegElems; ++j) {
        if ((live >> j) & 1u) {
            lo = fminf(lo, x[j]);
            hi = fmaxf(hi, x[j]);
            ++n;
        }
    }
    block_max_min_f(hi, lo, m, 4, lane, warp);
    cnt = block_sum_i(n, m, 4, lane, warp);
    below = 0;
    for (int pass = 0; pass < 8; ++pass) {
        if (lo == hi) {
            vstar = lo;
            if (kMass && pass > 0) {   // the mass passes keep no counts: the members left, counted once
                int nl = 0;
#pragma unroll
                for (int j = 0; j < kRegElems; ++j) nl += (live >> j) & 1u;
                cnt = block_sum_i(nl, m, 4, lane, warp);
            }
            return true;
        }
        const float scale = __fdiv_rn(256.0f, __fsub_rn(hi, lo));
        if (!(scale > 0.0f) || !(scale < pos_inf())) return false;
        uint32_t* bw = kMass ? &m.u.bins.m[0][0] : &m.u.bins.cnt[0];
        for (int i = tid; i < (kMass ? 2 : 1) * 256; i += kThreads) bw[i] = 0u;
        cbar();
#pragma unroll
        for (int j = 0; j < kRegElems; ++j) {
            if ((live >> j) & 1u) {
                const int b = min(255, static_cast<int>(__fmul_rn(__fsub_rn(x[j], lo), scale)));
                if (kMass) {
                    const unsigned long long f = __double2ull_rn(__dmul_rn(ev(j), kFix));   // <= 2^40
                    atomicAdd(&m.u.bins.m[0][b], static_cast<uint32_t>(f & 0xfffffull));
                    atomicAdd(&m.u.bins.m[1][b], static_cast<uint32_t>(f >> 20));
                } else {
                    atomicAdd(&m.u.bins.cnt[b], 1u);
                }
            }
        }
        cbar();
        if (warp == 0) {
            unsigned long long w8[8], loc = 0;
#pragma unroll
            for (int b = 0; b < 8; ++b) {
                const int bb = lane * 8 + b;
                w8[b] = kMass ? (static_cast<unsigned long long>(m.u.bins.m[0][bb]) +
                                 (static_cast<unsigned long long>(m.u.bins.m[1][bb]) << 20))
                              : static_cast<unsigned long long>(m.u.bins.cnt[bb]);
                loc += w8[b];
            }
            unsigned long long incl = loc;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned long long y = __shfl_up_sync(kFull, incl, o);
                if (lane >= o) incl += y;
            }
            unsigned long long acc = below + incl - loc;
            int found = -1;
            unsigned long long acc_before = 0;
            if (below + incl > target && acc <= target) {
#pragma unroll
                for (int b = 0; b < 8; ++b) {
                    const unsigned long long nxt = acc + w8[b];
                    if (found < 0 && nxt > target) {
                        found = lane * 8 + b;
                        acc_before = acc;
                    }
                    acc = nxt;
                }
            }
            const unsigned who = __ballot_sync(kFull, found >= 0);
            if (lane == 0) m.bc_i[0] = who ? 1 : 0;
            if (who) {
                const int src = __ffs(who) - 1;
                const int d = __shfl_sync(kFull, found, src);
                const unsigned long long ab = __shfl_sync(kFull, acc_before, src);
                if (lane == 0) {
                    m.bc_i[1] = d;
                    m.bc_i[2] = kMass ? 0 : static_cast<int>(m.u.bins.cnt[d]);
                    m.bc_u[0] = ab;
                }
            }
        }
        cbar();
        if (!m.bc_i[0]) return false;   // target at or past the total: no crossing
        const int bstar = m.bc_i[1];
        below = m.bc_u[0];
        cnt = m.bc_i[2];
        float nlo = pos_inf(), nhi = neg_inf();
#pragma unroll
        for (int j = 0; j < kRegElems; ++j) {
            if ((live >> j) & 1u) {
                const int b = min(255, static_cast<int>(__fmul_rn(__fsub_rn(x[j], lo), scale)));
                if (b != bstar) {
                    live &= ~(1u << j);
                } else {
                    nlo = fminf(nlo, x[j]);
                    nhi = fmaxf(nhi, x[j]);
                }
            }
        }
        block_max_min_f(nhi, nlo, m, 6, lane, warp);   // also orders this pass's reads before the next zeroing
        lo = nlo;
        hi = nhi;
    }
    return false;
}

// ---------------------------------------------------------------- general path, parallel (element threads)
// x[g * VW + e] is staged position (tid + 128 g) * VW + e, valid while (tid + 128 g) < nvec; the staged order is
// the index order.  `ecache` (shared or global memory, kRegElems * 128 doubles) keeps each value's softmax
// numerator at [j * 128 + tid] (0 for non-survivors).  Returns the sampled id, or -1 when a decision lies inside
// the error band.
template <int VW>
__device__ int general_parallel(const float (&x)[kRegElems], int nvec, const RowMap& mp, int V,
                                const DevOptions& o, double r, float mx, double* out_probs, double* ecache,
                                SmemMisc& m, int tid, int lane, int warp) {
    constexpr int G = kRegElems / VW;
    constexpr int FB = VW == 4 ? 10 : 11;           // bits per packed count field
    if (is_neg_inf(mx)) return -1;                  // all -inf: the replay reproduces the NaN behaviour
    uint32_t fin = 0;                               // bit j: finite value
#pragma unroll
    for (int j = 0; j < kRegElems; ++j)
        if (!is_neg_inf(x[j])) fin |= 1u << j;
    // ---- top-k threshold: the K-th largest value
    float kth = neg_inf();
    const int K = o.top_k;
    if (K > 0 && K < V) {
        const int F = block_sum_i(__popc(fin), m, 0, lane, warp);
        if (K <= F) {   // else the K-th largest is -inf and the cut keeps every finite value
            unsigned long long bl;
            int cnt;
            auto none = [](int) { return 0.0; };
            if (!binned_search<false>(x, fin, none, static_cast<unsigned long long>(F - K), m, tid, lane, warp, kth,
                                      bl, cnt))
                return -1;
        }
    }
    uint32_t surv = 0;
#pragma unroll
    for (int j = 0; j < kRegElems; ++j)
        if (((fin >> j) & 1u) && x[j] >= kth) surv |= 1u << j;
    // ---- softmax numerators of the survivors, total and count
    auto ev = [&](int j) -> double { return ecache[j * kThreads + tid]; };   // 0 for non-survivors
    double lsum = 0.0;
#pragma unroll
    for (int j = 0; j < kRegElems; ++j) {
        const double ej = ((surv >> j) & 1u) ? softmax_num(x[j], mx) : 0.0;
        ecache[j * kThreads + tid] = ej;
        lsum = __dadd_rn(lsum, ej);
    }
    const double total = block_sum_d(lsum, m, 0, lane, warp);
    const int nsurv = block_sum_i(__popc(surv), m, 1, lane, warp);
    const double eta = (8.0 * nsurv + 128.0) * kU;
    uint32_t removed = 0;   // bit j: element j removed by top-p
    if (o.top_p < 1.0f) {
        const double thr = static_cast<double>(__fsub_rn(1.0f, o.top_p));
        const double T = __dmul_rn(thr, total);
        const double before_last = __dsub_rn(total, 1.0);   // mass of every survivor but one max (e(max) = 1)
        const double band = __dmul_rn(eta, total);
        if (__dsub_rn(T, before_last) > band) {
            // the cut never fires before the last element: every survivor but the last of the order goes.  The
            // last is the max with the highest index; survivors below the max must have a strictly smaller
            // probability in the reference too.
            int li = -1;
            float below = neg_inf();
#pragma unroll
            for (int j = 0; j < kRegElems; ++j) {
                if ((surv >> j) & 1u) {
                    const int qv = tid + (j / VW) * kThreads;
                    if (x[j] == mx) li = max(li, mp.idx(qv * VW + (j % VW)));
                    else below = fmaxf(below, x[j]);
                }
            }
            li = block_max_i(li, m, 0, lane, warp);
            below = block_max_f(below, m, 0, lane, warp);
            if (!is_neg_inf(below) && !(softmax_num(below, mx) < 1.0 - 32.0 * kU)) return -1;
#pragma unroll
            for (int j = 0; j < kRegElems; ++j) {
                const int qv = tid + (j / VW) * kThreads;
                if (((surv >> j) & 1u) && mp.idx(qv * VW + (j % VW)) != li) removed |= 1u << j;
            }
        } else if (__dsub_rn(before_last, T) > band) {
            // the group x* holding the break element, by mass from the smallest value up
            const unsigned long long tfx = __double2ull_rn(__dmul_rn(T, kFix));
            float xs;
            unsigned long long below_fx;
            int ng;
            if (!binned_search<true>(x, surv, ev, tfx, m, tid, lane, warp, xs, below_fx, ng)) return -1;
            const double below = __dmul_rn(static_cast<double>(below_fx), 1.0 / kFix);
            // `below` sums masses rounded to 2^-40 each: within nsurv * 2^-41 of the exact sum, on top of the band
            const double bandm = __dadd_rn(band, static_cast<double>(nsurv + 1) * 0x1p-41);
            const double es = softmax_num(xs, mx);
            const double q = __ddiv_rn(__dsub_rn(T, below), es);
            if (!(q >= 0.0) || !(q < static_cast<double>(ng))) return -1;
            const int jrem = static_cast<int>(floor(q));   // group members removed (lowest ids first)
            const double last_removed = __dadd_rn(below, __dmul_rn(static_cast<double>(jrem), es));
            const double brk = __dadd_rn(below, __dmul_rn(static_cast<double>(jrem + 1), es));
            if (!(__dsub_rn(brk, T) > bandm)) return -1;
            if (last_removed > 0.0 && !(__dsub_rn(T, last_removed) > bandm)) return -1;
            // neighbours: the reference orders by probability, so the groups next to x* must be strictly apart
            float lo_n = neg_inf(), hi_n = pos_inf();
#pragma unroll
            for (int j = 0; j < kRegElems; ++j) {
                if ((surv >> j) & 1u) {
                    if (x[j] < xs) lo_n = fmaxf(lo_n, x[j]);
                    if (x[j] > xs) hi_n = fminf(hi_n, x[j]);
                }
            }
            block_max_min_f(lo_n, hi_n, m, 2, lane, warp);
            if (!is_neg_inf(lo_n) && !(softmax_num(lo_n, mx) < es * (1.0 - 32.0 * kU))) return -1;
            if (jrem > 0 && hi_n != pos_inf() && !(softmax_num(hi_n, mx) > es * (1.0 + 32.0 * kU))) return -1;
            // rank of each x* member in index order (packed per-vector counts, one block scan)
            unsigned long long packed = 0;
#pragma unroll
            for (int g = 0; g < G; ++g) {
                unsigned cg = 0;
#pragma unroll
                for (int t = 0; t < VW; ++t) {
                    const int j = g * VW + t;
                    cg += (((surv >> j) & 1u) && x[j] == xs) ? 1u : 0u;
                }
                packed |= static_cast<unsigned long long>(cg) << (FB * g);
            }
            unsigned long long pex, ptot;
            block_scan_u64(packed, m, 0, lane, warp, pex, ptot);
            const unsigned long long fmask = (1ull << FB) - 1;
            unsigned base_g = 0;
#pragma unroll
            for (int g = 0; g < G; ++g) {
                unsigned rk = base_g + static_cast<unsigned>((pex >> (FB * g)) & fmask);
#pragma unroll
                for (int t = 0; t < VW; ++t) {
                    const int j = g * VW + t;
                    if ((surv >> j) & 1u) {
                        if (x[j] < xs || (x[j] == xs && rk < static_cast<unsigned>(jrem))) removed |= 1u << j;
                        if (x[j] == xs) ++rk;
                    }
                }
                base_g += static_cast<unsigned>((ptot >> (FB * g)) & fmask);
            }
        } else {
            return -1;
        }
    }
    // ---- inverse-CDF draw over the kept ids in index order
    double c[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        c[g] = 0.0;
#pragma unroll
        for (int t = 0; t < VW; ++t) {
            const int j = g * VW + t;
            if (!((removed >> j) & 1u)) c[g] = __dadd_rn(c[g], ev(j));
        }
    }
    // per-vector exclusive prefix across threads, and the per-vector totals
    double ex[G], tot[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const double incl = warp_incl_d(c[g], lane);
        ex[g] = warp_excl_from_incl_d(incl, lane);
        if (lane == 31) m.red_v[warp][g] = incl;
    }
    cbar();
    double B = 0.0;
#pragma unroll
    for (int g = 0; g < G; ++g) {
        double base = 0.0, t = 0.0;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            const double v = m.red_v[w][g];
            if (w < warp) base = __dadd_rn(base, v);
            t = __dadd_rn(t, v);
        }
        ex[g] = __dadd_rn(ex[g], base);
        tot[g] = t;
        B = __dadd_rn(B, t);
    }
    const double rB = __dmul_rn(r, B);
    const double bandB = __dmul_rn(eta, B);
    int hit = -1, hits = 0;
    bool unsure = false;
    double run = 0.0;
#pragma unroll
    for (int g = 0; g < G; ++g) {
        double pre = __dadd_rn(run, ex[g]);
#pragma unroll
        for (int t = 0; t < VW; ++t) {
            const int j = g * VW + t;
            const double ej = ((removed >> j) & 1u) ? 0.0 : ev(j);
            if (ej > 0.0) {
                const double inc = __dadd_rn(pre, ej);
                if (inc > rB && !(pre > rB)) {
                    ++hits;
                    hit = mp.idx((tid + g * kThreads) * VW + t);
                    if (!(__dsub_rn(inc, rB) > bandB)) unsure = true;
                    if (pre > 0.0 && !(__dsub_rn(rB, pre) > bandB)) unsure = true;
                }
                pre = inc;
            }
        }
        run = __dadd_rn(run, tot[g]);
    }
    hits = block_sum_i(hits, m, 2, lane, warp);
    const bool any_unsure = cbar_or(unsure);
    if (hits != 1 || any_unsure) return -1;
    hit = block_max_i(hit, m, 3, lane, warp);
    if (out_probs) {
        for (int i = tid; i < V; i += kThreads) out_probs[i] = 0.0;
        cbar();
#pragma unroll
        for (int j = 0; j < kRegElems; ++j) {
            const int qv = tid + (j / VW) * kThreads;
            if (qv < nvec) {
                const int i = mp.idx(qv * VW + (j % VW));
                if (i < V) out_probs[i] = ((removed >> j) & 1u) ? 0.0 : __ddiv_rn(ev(j), B);
            }
        }
        cbar();
    }
    return hit;
}


// ---------------------------------------------------------------- candidate path (top-k <= 64)
constexpr double kFix52 = 4503599627370496.0;   // 2^52: candidate masses in fixed point (e <= 1, <= 128 values)

// ---------------------------------------------------------------- candidate replay (warp 0)
// The reference's sequential operations on the candidates (<= 128 survivors), every lane of one warp running the
// same chain on shuffled values.
__device__ __noinline__ int replay_candidates(const unsigned long long* ck, int C, int K, const DevOptions& o, double uniform,
                                 int V, double* out_probs, int* flags, int lane) {
    uint64_t key[4];   // descending value, ascending index
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        const int e = s * 32 + lane;
        key[s] = e < C ? ((static_cast<uint64_t>(~static_cast<uint32_t>(ck[e] >> 32)) << 32) |
                          static_cast<uint32_t>(ck[e]))
                       : ~0ull;
    }
    warp_sort<4>(key, lane);
    uint64_t kk = 0;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        const uint64_t v = shfl_u64(key[s], (K - 1) & 31);
        if (s == ((K - 1) >> 5)) kk = v;
    }
    const uint32_t kth_key = ~static_cast<uint32_t>(kk >> 32);
    int S = 0;
#pragma unroll
    for (int s = 0; s < 4; ++s)
        S += __popc(__ballot_sync(kFull, key[s] != ~0ull && (~static_cast<uint32_t>(key[s] >> 32)) >= kth_key));
    const float mx = okey_inv(~static_cast<uint32_t>(shfl_u64(key[0], 0) >> 32));
    // survivors are positions [0, S); re-sort them by index
    uint64_t k2[4];
#pragma unroll
    for (int s = 0; s < 4; ++s)
        k2[s] = (s * 32 + lane) < S ? ((static_cast<uint64_t>(static_cast<uint32_t>(key[s])) << 32) |
                                       ~static_cast<uint32_t>(key[s] >> 32))
                                    : ~0ull;
    warp_sort<4>(k2, lane);
    int idx[4];
    double p[4];
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        idx[s] = static_cast<int>(k2[s] >> 32);
        p[s] = (s * 32 + lane) < S ? softmax_num(okey_inv(static_cast<uint32_t>(k2[s])), mx) : 0.0;
    }
    double s1 = 0.0;   // Sampler.cs:58
#pragma unroll
    for (int s = 0; s < 4; ++s)
        for (int l = 0; l < 32 && s * 32 + l < S; ++l) s1 = __dadd_rn(s1, shfl_d(p[s], l));
#pragma unroll
    for (int s = 0; s < 4; ++s) p[s] = __ddiv_rn(p[s], s1);   // :60
    if (o.top_p < 1.0f) {   // :62-75
        const double thr = static_cast<double>(__fsub_rn(1.0f, o.top_p));
        uint64_t pk[4];
        uint32_t tag[4];
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            const int e = s * 32 + lane;
            pk[s] = e < S ? static_cast<uint64_t>(__double_as_longlong(p[s])) : ~0ull;
            tag[s] = static_cast<uint32_t>(e);   // index-order position
        }
        warp_sort_pair<4>(pk, tag, lane);
        double cum = 0.0;
        int m = S - 1;
        bool done = false;
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            for (int l = 0; l < 32 && !done; ++l) {
                const int j = s * 32 + l;
                if (j >= S - 1) {
                    done = true;
                    break;
                }
                cum = __dadd_rn(cum, __longlong_as_double(static_cast<long long>(shfl_u64(pk[s], l))));
                if (!(cum <= thr)) {
                    m = j;
                    done = true;
                }
            }
        }
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            const int j = s * 32 + lane;
            if (j < S) flags[tag[s]] = j < m ? 1 : 0;
        }
        __syncwarp();
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            const int e = s * 32 + lane;
            if (e < S && flags[e]) p[s] = 0.0;
        }
        __syncwarp();
        double s2 = 0.0;   // probs.Sum() (:73)
#pragma unroll
        for (int s = 0; s < 4; ++s)
            for (int l = 0; l < 32 && s * 32 + l < S; ++l) s2 = __dadd_rn(s2, shfl_d(p[s], l));
#pragma unroll
        for (int s = 0; s < 4; ++s) p[s] = __ddiv_rn(p[s], s2);   // :74
    }
    double acc = 0.0;   // inverse-CDF draw (:77-87)
    int last = 0, res = -1;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        for (int l = 0; l < 32 && s * 32 + l < S && res < 0; ++l) {
            const double v = shfl_d(p[s], l);
            const int id = __shfl_sync(kFull, idx[s], l);
            if (v <= 0.0) continue;
            acc = __dadd_rn(acc, v);
            last = id;
            if (uniform < acc) res = id;
        }
    }
    if (out_probs) {
        for (int i = lane; i < V; i += 32) out_probs[i] = 0.0;
        __syncwarp();
#pragma unroll
        for (int s = 0; s < 4; ++s)
            if (s * 32 + lane < S) out_probs[idx[s]] = p[s];
    }
    return res < 0 ? last : res;
}

// ---------------------------------------------------------------- element pass
// One pass over the staged row: transform every element into x[] (registers).  Sampling rows track each thread's
// two largest values; greedy rows the first maximum.  Vectors that no mask boundary, EOS rule or per-element
// penalty touches take the short path (temperature only).
template <int VW, bool kSample>
__device__ __forceinline__ void process_vectors(const unsigned char* sl, int nvec, const RowMap& mp,
                                                const RowCtx& c, int tid, float (&x)[kRegElems],
                                                float& tmax, float& tmax2, float& bestv, int& besti) {
    constexpr int G = kRegElems / VW;
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const int qv = tid + g * kThreads;
        if (qv < nvec) {
            float v[VW];
            load_vec<VW>(sl, qv, v);
            const int i0 = mp.idx(qv * VW);
            const uint32_t bits = c.pen_on ? pen_mask<VW>(c.flags, i0) : 0u;
            const bool slow = bits != 0u ||
                              static_cast<unsigned>(qv - c.slow_vlo) < static_cast<unsigned>(c.slow_vhi - c.slow_vlo) ||
                              qv == c.eos_vec;
#pragma unroll
            for (int e = 0; e < VW; ++e) {
                float t;
                if (slow)
                    t = transform(v[e], i0 + e, (bits >> e) & 1u, c);
                else
                    t = kSample ? __fmul_rn(v[e], c.inv_t) : v[e];
                x[g * VW + e] = t;
                if (kSample) {
                    tmax2 = fmaxf(tmax2, fminf(tmax, t));
                    tmax = fmaxf(tmax, t);
                } else if (t > bestv) {
                    bestv = t;
                    besti = i0 + e;
                }
            }
        } else {
#pragma unroll
            for (int e = 0; e < VW; ++e) x[g * VW + e] = neg_inf();
        }
    }
}

// Writes the register-resident row into gx[0, V) (every index into x is a compile-time constant, so x stays in
// registers).
template <int VW>
__device__ __forceinline__ void scatter_row(const float (&x)[kRegElems], int nvec, const RowMap& mp, int V,
                                            float* gx, int tid) {
#pragma unroll
    for (int j = 0; j < kRegElems; ++j) {
        const int qv = tid + (j / VW) * kThreads;
        if (qv < nvec) {
            const int i = mp.idx(qv * VW + (j % VW));
            if (i < V) gx[i] = x[j];
        }
    }
}

// Greedy: first index of the maximum over the 128 element threads (Sampler.cs:90-95).
__device__ int block_argmax(float bestv, int besti, SmemMisc& m, int lane, int warp) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(kFull, bestv, off);
        const int oi = __shfl_xor_sync(kFull, besti, off);
        if (ov > bestv || (ov == bestv && oi < besti)) {
            bestv = ov;
            besti = oi;
        }
    }
    if (lane == 0) {
        m.red_f[7][warp] = bestv;
        m.red_i[7][warp] = besti;
    }
    cbar();
    float bv = m.red_f[7][0];
    int bi = m.red_i[7][0];
    for (int w = 1; w < kWarps; ++w)
        if (m.red_f[7][w] > bv || (m.red_f[7][w] == bv && m.red_i[7][w] < bi)) {
            bv = m.red_f[7][w];
            bi = m.red_i[7][w];
        }
    return is_neg_inf(bv) ? 0 : bi;   // all -inf: the reference's scan never moves off index 0
}

// ---------------------------------------------------------------- producer warp (whole-row kernel)
// Plans the CTA's rows (CTA b takes entries b, b + gstride, ... of the deferred list) and streams each row's staged
// logits and history into the stage ring with bulk copies that complete on full_bar.  The row's RowMeta goes into
// metas[k % (2 * S)].
// The RowMeta of row r: where its data is, what to stage and how the element warps treat it.  `bytes` = the
// bytes its bulk copies bring into the stage (0 for a row that copies nothing), `esize` the logit size.
__device__ RowMeta plan_row(const LaunchParams& p, int r, uint32_t& bytes, int& esize) {
    RowMeta m;
    bytes = 0;
    esize = 4;
    int s = 0;
    for (int i = 1; i < p.n_segs; ++i)
        if (r >= p.seg[i].row_begin) s = i;
    const DevSegment& sg = p.seg[s];
    const int local = r - sg.row_begin;
    const int opt_raw = sg.opt_index ? sg.opt_index[local] : 0;
    const int V = sg.vocab;
    m.row = r;
    m.seg = s;
    m.opt_idx = opt_raw;
    m.step = sg.steps ? sg.steps[local] : 0x7fffffff;
    m.uniform = sg.uniforms ? sg.uniforms[local] : 0.0;
    int64_t hb = 0, he = 0;
    if (row_history(sg, local, hb, he) && (hb < 0 || he < hb)) {
        // device-memory offsets are checked here: report, and read no history
        atomicOr(p.err, kErrHistOffsets);
        hb = he = 0;
    }
    m.opt_ok = (opt_raw >= 0 && opt_raw < p.n_opts) ? 1 : 0;
    if (m.opt_ok) {
        m.opt = p.n_opts <= kInlineOptions ? p.inl_opts[opt_raw] : p.dev_opts[opt_raw];
    } else {
        m.opt = DevOptions{0, 0, 1.0f, 1.0f, 1.0f};
    }
    esize = sg.dtype == 0 ? 4 : 2;
    const int vsh = sg.dtype == 0 ? 2 : 3;   // log2 of the ids per 16-byte vector (no integer division per row)
    const int VWe = 1 << vsh;
    m.V = V;
    m.dtype = sg.dtype;
    m.kind = sg.kind;
    m.sup_lo = sg.sup_lo;
    m.sup_hi = sg.sup_hi;
    m.eos = sg.eos;
    m.eos_blocked = (sg.kind == 0 && m.step < sg.min_new) ? 1 : 0;
    m.pen_on = (m.opt_ok && sg.kind == 0 && m.opt.rep_penalty != 1.0f && he > hb) ? 1 : 0;
    m.pen_rcp = __drcp_rn(static_cast<double>(m.opt.rep_penalty));
    m.inv_t = __fdiv_rn(1.0f, m.opt.temperature);
    m.hist = sg.hist_ids ? sg.hist_ids + hb : nullptr;
    m.hist_len = static_cast<int32_t>(he - hb);
    m.out_id = sg.out_ids + local;
    m.out_probs = sg.out_probs ? sg.out_probs + static_cast<int64_t>(local) * V : nullptr;
    m.lo_al = V;
    m.hi_al = V;
    if (sg.kind == 0 && sg.sup_lo < sg.sup_hi) {
        const int la = ((sg.sup_lo + VWe - 1) >> vsh) << vsh;   // sup_lo, sup_hi are clamped to [0, V]
        const int ha = (sg.sup_hi >> vsh) << vsh;
        if (la < ha) {
            m.lo_al = la;
            m.hi_al = ha;
        }
    }
    const bool keep = sg.kind == 0 && sg.eos >= m.lo_al && sg.eos < m.hi_al && !m.eos_blocked;
    m.kvw = keep ? VWe : 0;
    m.kbase = keep ? (sg.eos >> vsh) << vsh : 0;   // keep: eos >= lo_al >= 0
    m.direct = sg.bulk_ok ? 0 : 1;
    m.hs_lo = 0;
    m.hs_hi = 0;
    if (m.pen_on && sg.hist_aligned && p.stage_hist_cap > 0) {
        int64_t a = (hb + 3) / 4 * 4;
        int64_t b = he / 4 * 4;
        if (b > a + p.stage_hist_cap) b = a + p.stage_hist_cap;
        if (b > a) {
            m.hs_lo = static_cast<int32_t>(a - hb);
            m.hs_hi = static_cast<int32_t>(b - hb);
        }
    }
    // staged vectors that may hold suppressed ids: positions [sup_lo, lo_al + kvw + (sup_hi - hi_al))
    m.slow_vlo = m.slow_vhi = 0;
    m.eos_vec = -1;
    if (sg.kind == 0) {
        if (sg.sup_lo < sg.sup_hi) {
            m.slow_vlo = sg.sup_lo >> vsh;
            m.slow_vhi = (m.lo_al + m.kvw + max(sg.sup_hi - m.hi_al, 0) + VWe - 1) >> vsh;
        }
        if (m.eos_blocked && sg.eos >= 0 && sg.eos < V) {
            const RowMap mp{m.lo_al, m.kvw, m.kbase, m.hi_al};
            const int ep = mp.pos(sg.eos);
            if (ep >= 0) m.eos_vec = ep >> vsh;
        }
    }
    m.row_ptr = static_cast<const unsigned char*>(sg.logits) +
                static_cast<int64_t>(local) * sg.row_stride * esize;
    if (m.opt_ok) {
        if (!m.direct) bytes += static_cast<uint32_t>((m.lo_al + m.kvw + V - m.hi_al) * esize);
        bytes += static_cast<uint32_t>(m.hs_hi - m.hs_lo) * 4u;
    }
    return m;
}

// Issues row m's bulk copies into stage `s` (the caller has armed full_bar[s] with their byte count).
__device__ __forceinline__ void issue_row(const LaunchParams& p, const RowMeta& m, int esize, unsigned char* log_dst,
                                          uint64_t* bar) {
    unsigned char* hist_dst = log_dst + p.stage_logit_bytes;
    if (!m.direct && m.opt_ok) {
        const int V = m.V;
        if (m.lo_al > 0) bulk_g2s(log_dst, m.row_ptr, static_cast<uint32_t>(m.lo_al * esize), bar);
        if (m.kvw > 0)
            bulk_g2s(log_dst + m.lo_al * esize, m.row_ptr + static_cast<int64_t>(m.kbase) * esize, 16u, bar);
        if (V > m.hi_al)
            bulk_g2s(log_dst + (m.lo_al + m.kvw) * esize, m.row_ptr + static_cast<int64_t>(m.hi_al) * esize,
                     static_cast<uint32_t>((V - m.hi_al) * esize), bar);
    }
    if (m.hs_hi > m.hs_lo && m.opt_ok)
        bulk_g2s(hist_dst, m.hist + m.hs_lo, static_cast<uint32_t>(m.hs_hi - m.hs_lo) * 4u, bar);
}

__device__ void produce_rows(const LaunchParams& p, int first, int gstride, int n_my, int lane, unsigned char* stages,
                             int stage_bytes, RowMeta* metas, uint64_t* full_bar, uint64_t* empty_bar,
                             const volatile uint32_t* progress, int* issued) {
    const int S_ = p.n_stages;
    bool alive = true;
    RingPos rp{0, 0};   // every lane advances it for every row
    for (int k0 = 0; k0 < n_my && alive; k0 += 32) {
        // lane j prepares the metadata of the CTA's row k0 + j
        const int kj = k0 + lane;
        RowMeta m;
        int esize = 4;
        uint32_t bytes = 0;
        if (kj < n_my) {
            int r = first + kj * gstride;
            r = min(max(p.deferred_rows[r], 0), p.total_rows - 1);
            m = plan_row(p, r, bytes, esize);
        }
        const int nb = (n_my - k0) < 32 ? (n_my - k0) : 32;
        for (int j = 0; j < nb; ++j) {
            bool ok = true;
            if (lane == j) {
                const int k = k0 + j;
                const int s = rp.s;
                if (rp.n > 0)
                    ok = mbar_wait_bounded(&empty_bar[s], static_cast<uint32_t>((rp.n - 1) & 1), p.wait_ns, progress);
                if (ok && m.row == p.test_stall_row) {
                    ok = false;   // test hook: this row's stage never completes, so the element warps' wait runs out
                } else if (ok) {
                    metas[rp.meta(S_)] = m;
                    fence_proxy_async();
                    mbar_arrive_expect_tx(&full_bar[s], bytes);
                    issue_row(p, m, esize, stages + static_cast<size_t>(s) * stage_bytes, &full_bar[s]);
                    *issued = k + 1;
                } else {
                    atomicOr(p.err, kErrTimeout);
                }
            }
            ok = __shfl_sync(kFull, ok ? 1 : 0, j) != 0;
            if (!ok) {
                alive = false;
                break;
            }
            rp.next(S_);
        }
    }
}

constexpr int kRankBuckets = 64;   // value buckets of the candidate counting sort

#include "vw_rowwarp.cuh"

// ---------------------------------------------------------------- whole-row kernel
// The rows the warp-per-row kernel deferred (the first deferred_count entries of deferred_rows): sampling rows with
// top-k off or K > 64, rows whose candidates overflowed, and rows of more than 3072 staged ids.  CTA b takes list
// entries b, b + grid, ...; each row is held in registers (24 values per thread) for the binned top-k / top-p
// searches, and rows whose decisions fall inside the error band are replayed in the reference's order.
// VWK as for row_warp_kernel: 4 / 8 when every segment holds fp32 / bf16 rows (one row path compiled in), 0 for a mix.
template <int VWK>
__global__ void __launch_bounds__(kBlockThreads, 3) whole_row_kernel(const __grid_constant__ LaunchParams p) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int S_ = p.n_stages;
    const int stage_bytes = p.stage_logit_bytes + p.stage_hist_cap * 4;
    unsigned char* stages = smem;
    RowMeta* metas = reinterpret_cast<RowMeta*>(smem + static_cast<size_t>(S_) * stage_bytes);   // 2 * S_ entries
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(metas + 2 * S_);
    uint64_t* empty_bar = full_bar + S_;
    uint8_t* flags = reinterpret_cast<uint8_t*>(empty_bar + S_);   // history flag map, a byte per id
    unsigned long long* ckey = reinterpret_cast<unsigned long long*>(flags + p.flag_bytes);
    SmemMisc& misc = *reinterpret_cast<SmemMisc*>(ckey + kCandCap);

    const int first = blockIdx.x;
    const int gstride = gridDim.x;
    // launched as a programmatic dependent of the warp-per-row kernel: wait until that grid has finished and its
    // deferred-row list is visible
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int n_rows = min(static_cast<int>(*reinterpret_cast<volatile uint32_t*>(p.deferred_count)), p.total_rows);
    const int n_my = first < n_rows ? (n_rows - 1 - first) / gstride + 1 : 0;
    // nothing deferred: the counters are already zero, so no CTA has anything to do
    if (n_rows == 0) return;

    if (tid == 0) {
        for (int s = 0; s < S_; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        fence_mbar_init();
        misc.issued = 0;
        misc.progress = 0;
    }
    for (int i = tid; i < p.flag_bytes / 16; i += blockDim.x) reinterpret_cast<uint4*>(flags)[i] = make_uint4(0, 0, 0, 0);
    __syncthreads();

    if (warp == kProducerWarp) {
        // ================= producer warp: plans rows and issues the bulk copies =================
        produce_rows(p, first, gstride, n_my, lane, stages, stage_bytes, metas, full_bar, empty_bar,
                               &misc.progress, &misc.issued);
        return;
    }

    // ================= element warps =================
    uint32_t st_greedy = 0, st_general = 0, st_general_exact = 0, st_large = 0;
    RingPos rp{0, 0};
    for (int k = 0; k < n_my; ++k, rp.next(S_)) {
        const int s = rp.s;
        unsigned char* sl = stages + static_cast<size_t>(s) * stage_bytes;
        const bool ok = mbar_wait_bounded(&full_bar[s], static_cast<uint32_t>(rp.n & 1), p.wait_ns);
        if (cbar_or(!ok)) {
            if (tid == 0) {
                atomicOr(p.err, kErrTimeout);
                // drain: wait (bounded) for every copy the producer issued after this row
                const int issued = *reinterpret_cast<volatile int*>(&misc.issued);
                for (int kk = k; kk < issued; ++kk)
                    mbar_wait_bounded(&full_bar[kk % S_], static_cast<uint32_t>((kk / S_) & 1), p.wait_ns);
            }
            cbar();
            break;
        }
        const RowMeta& m = metas[rp.meta(S_)];
        const int32_t* sh = reinterpret_cast<const int32_t*>(sl + p.stage_logit_bytes);
        const int V = m.V;
        const int dtype = VWK == 4 ? 0 : VWK == 8 ? 1 : m.dtype;
        const int VWe = dtype == 0 ? 4 : 8;
        const RowMap mp{m.lo_al, m.kvw, m.kbase, m.hi_al};
        const int NA = m.lo_al + m.kvw + (V - m.hi_al);
        const int nvec = (NA + VWe - 1) >> (dtype == 0 ? 2 : 3);   // bulk-copied rows have NA % VWe == 0
        double* out_probs = m.out_probs;

        if (!m.opt_ok) {
            cbar();
            if (tid == 0) {
                atomicOr(p.err, kErrBadOption);
                *m.out_id = -1;
                mbar_arrive(&empty_bar[s]);
                ++misc.progress;
            }
            continue;
        }
        const DevOptions o = m.opt;

        // ---- unaligned rows: the element warps stage the active ids themselves
        if (m.direct) {
            for (int q = tid; q < nvec * VWe; q += kThreads) {
                const int i = mp.idx(q);
                if (dtype == 0)
                    reinterpret_cast<float*>(sl)[q] = i < V ? reinterpret_cast<const float*>(m.row_ptr)[i] : neg_inf();
                else   // padding past V reads as bf16 -inf
                    reinterpret_cast<uint16_t*>(sl)[q] =
                        i < V ? reinterpret_cast<const uint16_t*>(m.row_ptr)[i] : 0xff80u;
            }
        }

        // ---- repetition penalty (Sampler.cs:25-33): Distinct() through a flag byte per id (plain stores); the
        //      element pass applies the penalty to every element whose flag is set
        if (m.pen_on) {
            bool bad = false;
            const int nst = m.hs_hi - m.hs_lo;
            for (int c4 = tid; c4 < nst / 4; c4 += kThreads) {
                const int4 hv = reinterpret_cast<const int4*>(sh)[c4];
                const int ids[4] = {hv.x, hv.y, hv.z, hv.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if (static_cast<unsigned>(ids[j]) < static_cast<unsigned>(V))
                        flags[ids[j]] = 1;
                    else
                        bad = true;
                }
            }
            // ids outside the staged span, [0, hs_lo) and [hs_hi, len), from global memory: four independent
            // loads per thread in flight
            const int rest = m.hist_len - nst;
            for (int q0 = tid; q0 < rest; q0 += 4 * kThreads) {
                int ids[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int q = q0 + j * kThreads;
                    ids[j] = q < rest ? m.hist[q < m.hs_lo ? q : q - m.hs_lo + m.hs_hi] : 0;
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if (q0 + j * kThreads >= rest) continue;
                    if (static_cast<unsigned>(ids[j]) < static_cast<unsigned>(V))
                        flags[ids[j]] = 1;
                    else
                        bad = true;
                }
            }
            if (bad) atomicOr(p.err, kErrHistRange);
        }
        if (m.pen_on || m.direct) cbar();

        RowCtx c;
        c.vocab = V;
        c.kind = m.kind;
        c.sup_lo = m.sup_lo;
        c.sup_hi = m.sup_hi;
        c.eos = m.eos;
        c.eos_blocked = m.eos_blocked != 0;
        c.pen_on = m.pen_on != 0;
        c.pen = o.rep_penalty;
        c.pen_rcp = m.pen_rcp;
        c.sample = o.do_sample != 0;
        c.inv_t = m.inv_t;
        c.flags = flags;
        c.slow_vlo = m.slow_vlo;
        c.slow_vhi = m.slow_vhi;
        c.eos_vec = m.eos_vec;

        char* gbase = p.gscratch + static_cast<int64_t>(blockIdx.x) * p.gscratch_stride;
        const int vpad = (max(p.vmax, kRegElems * kThreads) + 31) & ~31;
        float* gx = reinterpret_cast<float*>(gbase);
        double* gp = reinterpret_cast<double*>(gbase + static_cast<int64_t>(vpad) * 4);
        uint4* gs = reinterpret_cast<uint4*>(gbase + static_cast<int64_t>(vpad) * 12);
        int sort_n = 1;
        while (sort_n < V) sort_n <<= 1;

        const bool big = nvec > kThreads * (kRegElems / VWe);
        if (big) {
            // ---- rows with more than 3072 active ids: transform into global scratch, exact path
            float tmax = neg_inf(), bestv = neg_inf();
            int besti = 0x7fffffff;
            for (int i = tid; i < V; i += kThreads) gx[i] = neg_inf();
            cbar();
            for (int qv = tid; qv < nvec; qv += kThreads) {
                const int q0 = qv * VWe;
                const int i0 = mp.idx(q0);
                for (int e = 0; e < VWe && i0 + e < V; ++e) {
                    const float t = transform(load_elem(sl, q0 + e, dtype), i0 + e, flags[i0 + e] != 0, c);
                    gx[i0 + e] = t;
                    tmax = fmaxf(tmax, t);
                    if (t > bestv) {
                        bestv = t;
                        besti = i0 + e;
                    }
                }
            }
            cbar();
            if (tid == 0) mbar_arrive(&empty_bar[s]);
            if (m.pen_on)
                for (int i = tid; i < p.flag_bytes / 16; i += kThreads) reinterpret_cast<uint4*>(flags)[i] = make_uint4(0, 0, 0, 0);
            int res;
            if (!c.sample) {
                res = block_argmax(bestv, besti, misc, lane, warp);
                if (out_probs)
                    for (int i = tid; i < V; i += kThreads) out_probs[i] = 0.0;
            } else {
                const float mx = block_max_f(tmax, misc, 0, lane, warp);
                res = exact_block_path(c, o, m.uniform, mx, gx, gp, gs, sort_n, out_probs, misc, tid);
            }
            if (tid == 0) {
                *m.out_id = res;
                ++misc.progress;
            }
            ++st_large;
            cbar();
            continue;
        }

        float x[kRegElems];
        float tmax = neg_inf(), tmax2 = neg_inf();   // the two largest values of this thread
        float bestv = neg_inf();
        int besti = 0x7fffffff;
        if (c.sample) {
            if (dtype == 0)
                process_vectors<4, true>(sl, nvec, mp, c, tid, x, tmax, tmax2, bestv, besti);
            else
                process_vectors<8, true>(sl, nvec, mp, c, tid, x, tmax, tmax2, bestv, besti);
        } else {
            if (dtype == 0)
                process_vectors<4, false>(sl, nvec, mp, c, tid, x, tmax, tmax2, bestv, besti);
            else
                process_vectors<8, false>(sl, nvec, mp, c, tid, x, tmax, tmax2, bestv, besti);
        }
        cbar();   // the stage has been read
        if (m.pen_on)
            for (int i = tid; i < p.flag_bytes / 16; i += kThreads) reinterpret_cast<uint4*>(flags)[i] = make_uint4(0, 0, 0, 0);
        bool released = false;
        auto release = [&]() {   // hand the stage back to the producer (after a cbar)
            if (!released && tid == 0) mbar_arrive(&empty_bar[s]);
            released = true;
        };

        if (!c.sample) {
            release();
            const int res = block_argmax(bestv, besti, misc, lane, warp);
            if (out_probs)
                for (int i = tid; i < V; i += kThreads) out_probs[i] = 0.0;
            if (tid == 0) {
                *m.out_id = res;
                ++misc.progress;
            }
            ++st_greedy;
            continue;
        }

        {
            const float mx = block_max_f(tmax, misc, 0, lane, warp);
            // numerator cache: the consumed stage when it is large enough, else this CTA's global scratch
            const bool in_stage = !released && stage_bytes >= kRegElems * kThreads * 8;
            double* ecache = in_stage ? reinterpret_cast<double*>(sl) : gp;
            if (!in_stage) release();
            int res = -1;
            if (!p.force_exact)
                res = dtype == 0 ? general_parallel<4>(x, nvec, mp, V, o, m.uniform, mx, out_probs, ecache, misc, tid, lane, warp)
                                 : general_parallel<8>(x, nvec, mp, V, o, m.uniform, mx, out_probs, ecache, misc, tid, lane, warp);
            cbar();
            release();
            if (res >= 0) ++st_general;
            if (res < 0) {
                ++st_general_exact;
                for (int i = tid; i < V; i += kThreads) gx[i] = neg_inf();
                cbar();
                if (dtype == 0)
                    scatter_row<4>(x, nvec, mp, V, gx, tid);
                else
                    scatter_row<8>(x, nvec, mp, V, gx, tid);
                cbar();
                res = exact_block_path(c, o, m.uniform, mx, gx, gp, gs, sort_n, out_probs, misc, tid);
            }
            if (tid == 0) *m.out_id = res;
        }
        if (tid == 0) ++misc.progress;
    }
    if (tid == 0) {
        // the last whole-row CTA to finish clears the deferred list for the next call
        __threadfence();
        if (atomicAdd(p.done_count, 1u) == gridDim.x - 1) {
            *reinterpret_cast<volatile uint32_t*>(p.deferred_count) = 0u;
            *reinterpret_cast<volatile uint32_t*>(p.done_count) = 0u;
            __threadfence();
        }
    }
    if (tid == 0 && p.stats) {
        const uint32_t v[4] = {st_greedy, st_general, st_general_exact, st_large};
        const int idx[4] = {kStatGreedy, kStatGeneral, kStatGeneralReplayed, kStatLarge};
        for (int i = 0; i < 4; ++i)
            if (v[i]) atomicAdd(&p.stats[idx[i]], static_cast<unsigned long long>(v[i]));
    }
}

// ---------------------------------------------------------------- Sampler.ApplyRepetitionPenalty
__global__ void __launch_bounds__(256) penalty_kernel(float* logits, int vocab, const int32_t* hist,
                                                      int64_t hist_len, float penalty, unsigned* err) {
    extern __shared__ uint32_t bm[];
    const int words = (vocab + 31) / 32;
    for (int i = threadIdx.x; i < words; i += blockDim.x) bm[i] = 0u;
    __syncthreads();
    bool bad = false;
    for (int64_t j = threadIdx.x; j < hist_len; j += blockDim.x) {
        const int id = hist[j];
        if (static_cast<unsigned>(id) >= static_cast<unsigned>(vocab)) {
            bad = true;
            continue;
        }
        const uint32_t bit = 1u << (id & 31);
        const uint32_t old = atomicOr(&bm[id >> 5], bit);
        if (!(old & bit)) {   // first occurrence: Distinct()
            const float s = logits[id];
            logits[id] = s < 0.0f ? __fmul_rn(s, penalty) : __fdiv_rn(s, penalty);
        }
    }
    if (bad) atomicOr(err, kErrHistRange);
}

// ---------------------------------------------------------------- exp diagnostic
// The sampler's exp (libm_exp) and CUDA's exp over an array.
__global__ void __launch_bounds__(256) exp_diag_kernel(const double* x, int64_t n, double* y_libm, double* y_cuda) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const double v = x[i];
        if (y_libm) y_libm[i] = libm_exp(v);
        if (y_cuda) y_cuda[i] = exp(v);
    }
}

}  // namespace

cudaError_t launch_exp_diagnostic(const double* x, int64_t n, double* y_libm, double* y_cuda, int sm_count,
                                  cudaStream_t stream) {
    const int64_t blocks = std::min<int64_t>((n + 255) / 256, static_cast<int64_t>(sm_count) * 8);
    if (blocks > 0) exp_diag_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(x, n, y_libm, y_cuda);
    return cudaGetLastError();
}

// ---------------------------------------------------------------- host-side launch helpers
size_t sampler_smem_bytes(const LaunchParams& p) {
    const size_t stage = static_cast<size_t>(p.stage_logit_bytes) + static_cast<size_t>(p.stage_hist_cap) * 4;
    size_t b = stage * p.n_stages;
    b += sizeof(RowMeta) * 2 * p.n_stages;
    b += sizeof(uint64_t) * (2 * p.n_stages);
    b += static_cast<size_t>(p.flag_bytes);
    b += sizeof(unsigned long long) * kCandCap;
    b += sizeof(SmemMisc);
    return b;
}

int64_t sampler_gscratch_stride(int vmax) {
    const int64_t vpad = (std::max(vmax, kRegElems * kThreads) + 31) & ~31;
    int64_t sort_n = 1;
    while (sort_n < vmax) sort_n <<= 1;
    int64_t b = vpad * 4 + vpad * 8 + sort_n * 16;
    return (b + 255) & ~static_cast<int64_t>(255);
}

namespace {
// Resident CTAs per SM of fns[0] at `threads` x `smem`; raises the dynamic shared-memory limit of every instance in
// fns (they share their resources) on the current device first when it needs more than the default 48 KB (once per
// device and size).
int ctas_per_sm(const void* const (&fns)[3], int which, int threads, size_t smem) {
    constexpr int kMaxDevices = 64;
    static std::mutex mu;
    static size_t configured[kMaxDevices][2] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
    if (smem > 48 * 1024) {
        std::lock_guard<std::mutex> lock(mu);
        if (smem > configured[dev][which]) {
            for (const void* fn : fns)
                if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
                    cudaSuccess)
                    return 0;
            configured[dev][which] = smem;
        }
    }
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fns[0], threads, smem) != cudaSuccess) return 0;
    return n;
}
}  // namespace

bool plan_launch(LaunchParams& p, int sm_count, int max_grid_general, LaunchPlan* plan) {
    const void* const fw[3] = {reinterpret_cast<const void*>(&row_warp_kernel<0>),
                               reinterpret_cast<const void*>(&row_warp_kernel<4>),
                               reinterpret_cast<const void*>(&row_warp_kernel<8>)};
    const void* const fg[3] = {reinterpret_cast<const void*>(&whole_row_kernel<0>),
                               reinterpret_cast<const void*>(&whole_row_kernel<4>),
                               reinterpret_cast<const void*>(&whole_row_kernel<8>)};
    // the whole-row kernel's stage count: the one that keeps the most of its CTAs resident (ties: the deeper ring)
    int best_stages = 0, best_cg = 0;
    for (int stages = kStages; stages >= 2; --stages) {
        p.n_stages = stages;
        const int cg = ctas_per_sm(fg, 1, kBlockThreads, sampler_smem_bytes(p));
        if (cg > best_cg) {
            best_stages = stages;
            best_cg = cg;
        }
    }
    if (best_stages == 0) return false;
    p.n_stages = best_stages;
    plan->smem_cand = static_cast<size_t>(kRwWarps) * rw_warp_bytes(p.vmax);
    const int cw = ctas_per_sm(fw, 0, kRwWarps * 32, plan->smem_cand);
    if (cw == 0) return false;
    plan->smem_general = sampler_smem_bytes(p);
    const int64_t warps_needed = (static_cast<int64_t>(p.total_rows) + kRwWarps - 1) / kRwWarps;
    plan->grid = static_cast<int>(std::min<int64_t>(warps_needed, static_cast<int64_t>(sm_count) * cw));
    plan->grid_general = static_cast<int>(std::min<int64_t>(
        {static_cast<int64_t>(p.total_rows), static_cast<int64_t>(sm_count) * best_cg,
         static_cast<int64_t>(max_grid_general)}));
    return true;
}

cudaError_t launch_sampler(const LaunchParams& p, const LaunchPlan& plan, cudaStream_t stream) {
    // one row path compiled into the kernels when every segment has the same dtype
    bool all_f32 = true, all_bf16 = true;
    for (int i = 0; i < p.n_segs; ++i) {
        all_f32 = all_f32 && p.seg[i].dtype == 0;
        all_bf16 = all_bf16 && p.seg[i].dtype != 0;
    }
    cudaError_t e;
    {   // a programmatic dependent of the stream's previous kernel (the kernel waits for it before reading anything)
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(plan.grid);
        cfg.blockDim = dim3(kRwWarps * 32);
        cfg.dynamicSmemBytes = plan.smem_cand;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        e = all_f32 ? cudaLaunchKernelEx(&cfg, row_warp_kernel<4>, p)
                    : all_bf16 ? cudaLaunchKernelEx(&cfg, row_warp_kernel<8>, p) : cudaLaunchKernelEx(&cfg, row_warp_kernel<0>, p);
        if (e != cudaSuccess) return e;
    }
    // programmatic dependent launch: the whole-row grid is scheduled while the candidate grid drains, instead of
    // after it (its kernel waits for the first grid's completion before reading the deferred list)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(plan.grid_general);
    cfg.blockDim = dim3(kBlockThreads);
    cfg.dynamicSmemBytes = plan.smem_general;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = all_f32 ? cudaLaunchKernelEx(&cfg, whole_row_kernel<4>, p)
                : all_bf16 ? cudaLaunchKernelEx(&cfg, whole_row_kernel<8>, p) : cudaLaunchKernelEx(&cfg, whole_row_kernel<0>, p);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

cudaError_t launch_apply_penalty(float* logits, int vocab, const int32_t* hist, int64_t hist_len, float penalty,
                                 unsigned* err, cudaStream_t stream) {
    const size_t smem = sizeof(uint32_t) * ((vocab + 31) / 32);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(penalty_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    penalty_kernel<<<1, 256, smem, stream>>>(logits, vocab, hist, hist_len, penalty, err);
    return cudaGetLastError();
}

}  // namespace vw

namespace vw {
namespace {
static_assert(sizeof(SmemMisc) % 16 == 0, "SmemMisc alignment");
}  // namespace
}  // namespace vw
