// vw_sampler.cu -- fused token-sampling kernel for sm_100a (B200).
//
// One warp-group (128 threads, "compute warps") samples one logits row at a time; a fifth "producer" warp
// streams the next rows into a shared-memory ring with cp.async.bulk (TMA bulk copies) completing on mbarriers,
// so HBM reads overlap the per-row work.  CTAs are persistent: CTA b takes rows b, b + grid, b + 2 grid, ...
//
// Per row, in the order of the reference (src/Voxwerk/Talker/Sampler.cs, TalkerGenerator.cs):
//   1. repetition penalty (talker rows; Sampler.cs:25-33): history ids -> a V-bit shared bitmap (Distinct());
//      each element whose bit is set becomes s < 0 ? s * p : s / p in fp32.  The IEEE quotient s / p is formed
//      as fp32(fp64(s) * RN64(1/p)); the fp64 product is within 2^-52 relative of s/p while no fp32 rounding
//      midpoint lies closer than 2^-49 relative to a quotient of two fp32 values, so both round the same way.
//   2. suppress mask (talker rows; TalkerGenerator.cs:247-248): ids [lo, hi) except EOS, and EOS while
//      t < min_new_tokens, become -inf.  The suppressed span is never read from HBM.
//   3. greedy rows: first index of the maximum (Sampler.cs:90-95).
//   4. temperature: x * fp32(1/T) (Sampler.cs:39-40).
//   5. top-k (Sampler.cs:42-49): every value >= the K-th largest survives (ties kept).  Candidates are the
//      values >= tau, where tau = min over the 4 warps of the ceil(K/4)-th largest lane maximum (so >= K values
//      are >= tau and the K-th largest is >= tau); one warp sorts the candidates (bitonic, 4 per lane).
//   6. softmax in fp64 over the survivors, the fp64 sum taken sequentially in index order (Sampler.cs:51-60),
//      top-p over the (prob, index)-ascending order with the reference's cumulative rule (:62-75) and the
//      inverse-CDF draw against the caller's uniform (:77-87).  These sums are order-dependent roundings, so
//      one warp replays them in the reference's order (every lane runs the same chain on shuffled values).
// Rows the small path cannot take (top-k off or K > 64, > 128 candidates, > 64 survivors, > 3072 active ids)
// take the general path: the same steps over the whole row in per-CTA global scratch.
//
// Compile with -fmad=false: no multiply-add may be contracted; every rounding step is explicit (_rn
// intrinsics) to match the reference's separately rounded fp32 / fp64 operations.

#include <cstdint>
#include <cuda_runtime.h>

#include "vw_internal.h"

namespace vw {
namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kMetaBytes = 128;
constexpr int kKeepBytes = 16;
constexpr uint64_t kWaitLimitNs = 2000000000ull;   // bounded mbarrier waits: 2 s

struct RowMeta {
    double uniform;
    int64_t hist_begin;   // absolute offset into the segment's hist_ids
    int32_t row;          // global row index
    int32_t seg, local, step, hist_len;
    int32_t hs_lo, hs_hi; // history ids [hs_lo, hs_hi) (relative to hist_begin) are staged in shared memory
    int32_t lo_al, hi_al; // staged logits: ids [0, lo_al) then [hi_al, V), packed
    int32_t keep;         // the 16-byte vector holding EOS is staged separately
    int32_t direct;       // logits were not bulk-copied: the compute warps load them
    int32_t pen_on;       // repetition penalty active
    int32_t opt_ok;       // option index valid
    DevOptions opt;
};
static_assert(sizeof(RowMeta) <= kMetaBytes, "RowMeta too large");

struct SmemMisc {
    float tau_w[kWarps];
    float red_v[kWarps];
    int32_t red_i[kWarps];
    uint32_t cand_count;
    int32_t decision;     // small path result (>= 0) or -1: take the general path
    int32_t issued;       // rows the producer has issued (for the timeout drain)
    int32_t pad;
    double bcast_d;
    int32_t bcast_i;
    int32_t pad2;
    uint32_t hist256[256];
    int32_t flags[kSmallSurvivors];
};

struct Cand {
    float x;
    int32_t idx;
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
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Waits for the phase with `parity` to complete; gives up after kWaitLimitNs and returns false.
__device__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (global_ns() - t0 > kWaitLimitNs) return false;
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
// Barrier among the 128 compute threads (named barrier 1; the producer warp never joins it).
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
__device__ __forceinline__ float neg_inf() { return __int_as_float(0xff800000); }
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
    const uint32_t* bitmap;
};

// penalty (Sampler.cs:31) -> mask (TalkerGenerator.cs:247-248) -> temperature (Sampler.cs:40)
__device__ __forceinline__ float transform(float v, int idx, uint32_t bits, const RowCtx& c) {
    if (c.pen_on && ((bits >> (idx & 31)) & 1u)) {
        v = v < 0.0f ? __fmul_rn(v, c.pen) : __double2float_rn(__dmul_rn(static_cast<double>(v), c.pen_rcp));
    }
    if (c.kind == 0) {
        const bool masked = (idx >= c.sup_lo && idx < c.sup_hi && idx != c.eos) || (idx == c.eos && c.eos_blocked);
        if (masked) v = neg_inf();
    }
    if (c.sample) v = __fmul_rn(v, c.inv_t);
    return v;
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

// ---------------------------------------------------------------- block reductions (compute warps)
// Max over the 128 compute threads.  Uses misc.red_v; one cbar.
__device__ float block_max(float v, SmemMisc& misc, int lane, int warp) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
    if (lane == 0) misc.red_v[warp] = v;
    cbar();
    float r = misc.red_v[0];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) r = fmaxf(r, misc.red_v[w]);
    return r;
}

// ---------------------------------------------------------------- general path (all 128 compute threads)
// gx[0, V) holds the transformed row (suppressed ids = -inf).  Returns the sampled id in every thread.
__device__ int general_path(const RowCtx& c, const DevOptions& o, double r, float mx, float* gx, double* gp,
                            uint4* gs, int sort_n, double* out_probs, SmemMisc& misc, int tid) {
    const int V = c.vocab;
    if (is_neg_inf(mx)) {
        // Every logit is -inf: the reference's probabilities are 0/0 = NaN, the draw never fires and it
        // returns the last index (Sampler.cs:80-87).
        if (out_probs)
            for (int i = tid; i < V; i += kThreads) out_probs[i] = 0.0;
        return V - 1;
    }
    // ---- top-k threshold: the K-th largest of the V values (radix select over order-preserving keys)
    float kth = neg_inf();
    const int K = o.top_k;
    if (K > 0 && K < V) {
        uint32_t prefix = 0, pmask = 0;
        int need = K;
        for (int shift = 24; shift >= 0; shift -= 8) {
            for (int b = tid; b < 256; b += kThreads) misc.hist256[b] = 0;
            cbar();
            for (int i = tid; i < V; i += kThreads) {
                const uint32_t k = okey(gx[i]);
                if ((k & pmask) == prefix) atomicAdd(&misc.hist256[(k >> shift) & 255u], 1u);
            }
            cbar();
            if (tid == 0) {
                int d = 255;
                for (; d > 0; --d) {
                    const int h = static_cast<int>(misc.hist256[d]);
                    if (need <= h) break;
                    need -= h;
                }
                misc.bcast_i = d;
                misc.bcast_d = static_cast<double>(need);
            }
            cbar();
            const uint32_t d = static_cast<uint32_t>(misc.bcast_i);
            need = static_cast<int>(misc.bcast_d);
            prefix |= d << shift;
            pmask |= 255u << shift;
            cbar();
        }
        kth = okey_inv(prefix);
    }
    // ---- softmax numerators (Sampler.cs:55-58): exp(fp64(fp32(x - max))) for survivors, 0 otherwise
    for (int i = tid; i < V; i += kThreads) {
        const float x = gx[i];
        gp[i] = (!is_neg_inf(x) && x >= kth) ? exp(static_cast<double>(__fsub_rn(x, mx))) : 0.0;
    }
    cbar();
    if (tid == 0) {   // sequential fp64 sum in index order (Sampler.cs:58)
        double s = 0.0;
        for (int i = 0; i < V; ++i) {
            const double v = gp[i];
            if (v != 0.0) s = __dadd_rn(s, v);
        }
        misc.bcast_d = s;
    }
    cbar();
    {
        const double s1 = misc.bcast_d;
        for (int i = tid; i < V; i += kThreads) gp[i] = __ddiv_rn(gp[i], s1);   // :60
    }
    cbar();
    if (o.top_p < 1.0f) {   // Sampler.cs:62-75
        const double thr = static_cast<double>(__fsub_rn(1.0f, o.top_p));
        for (int i = tid; i < sort_n; i += kThreads) {
            uint4 it;
            if (i < V) {
                const unsigned long long b = static_cast<unsigned long long>(__double_as_longlong(gp[i]));
                it = make_uint4(static_cast<uint32_t>(b), static_cast<uint32_t>(b >> 32), static_cast<uint32_t>(i), 0u);
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
                const double v = __longlong_as_double(static_cast<long long>((static_cast<uint64_t>(it.y) << 32) | it.x));
                if (v == 0.0) continue;   // adds 0 and removes an id that is already 0
                cum = __dadd_rn(cum, v);
                if (!(cum <= thr)) {
                    m = j;
                    break;
                }
            }
            misc.bcast_i = m;
        }
        cbar();
        {
            const int m = misc.bcast_i;
            for (int j = tid; j < m; j += kThreads) gp[gs[j].z] = 0.0;
        }
        cbar();
        if (tid == 0) {   // probs.Sum() in index order (:73)
            double s = 0.0;
            for (int i = 0; i < V; ++i) {
                const double v = gp[i];
                if (v != 0.0) s = __dadd_rn(s, v);
            }
            misc.bcast_d = s;
        }
        cbar();
        {
            const double s2 = misc.bcast_d;
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
        misc.bcast_i = res < 0 ? last : res;
    }
    if (out_probs)
        for (int i = tid; i < V; i += kThreads) out_probs[i] = gp[i];
    cbar();
    const int res = misc.bcast_i;
    cbar();
    return res;
}

// ---------------------------------------------------------------- small path (one warp)
// Candidates (x, idx) in `cand[0, C)`, C <= kCandCap.  Returns the sampled id, or -1 if the survivors
// exceed kSmallSurvivors.  Runs on warp 0 only.
__device__ int small_path(const Cand* cand, int C, const DevOptions& o, double r, double* out_probs,
                          SmemMisc& misc, int lane) {
    // descending value, ascending index
    uint64_t key[4];
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        const int e = s * 32 + lane;
        if (e < C) {
            const Cand cd = cand[e];
            key[s] = (static_cast<uint64_t>(~okey(cd.x)) << 32) | static_cast<uint32_t>(cd.idx);
        } else {
            key[s] = ~0ull;
        }
    }
    warp_sort<4>(key, lane);
    const int K = o.top_k;
    const int ks = (K - 1) >> 5, kl = (K - 1) & 31;
    uint64_t kk = 0;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        const uint64_t v = shfl_u64(key[s], kl);
        if (s == ks) kk = v;
    }
    const uint32_t kth_key = ~static_cast<uint32_t>(kk >> 32);
    int S = 0;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        const bool surv = key[s] != ~0ull && (~static_cast<uint32_t>(key[s] >> 32)) >= kth_key;
        S += __popc(__ballot_sync(kFull, surv));
    }
    if (S > kSmallSurvivors) return -1;
    const float mx = okey_inv(~static_cast<uint32_t>(shfl_u64(key[0], 0) >> 32));

    // survivors (positions [0, S)) re-sorted by index, carrying the value key
    uint64_t k2[2];
#pragma unroll
    for (int s = 0; s < 2; ++s) {
        const int e = s * 32 + lane;
        k2[s] = e < S ? ((static_cast<uint64_t>(static_cast<uint32_t>(key[s])) << 32) | ~static_cast<uint32_t>(key[s] >> 32))
                      : ~0ull;
    }
    warp_sort<2>(k2, lane);
    int idx[2];
    double p[2];
#pragma unroll
    for (int s = 0; s < 2; ++s) {
        const int e = s * 32 + lane;
        idx[s] = static_cast<int>(k2[s] >> 32);
        const float x = okey_inv(static_cast<uint32_t>(k2[s]));
        p[s] = e < S ? exp(static_cast<double>(__fsub_rn(x, mx))) : 0.0;   // Sampler.cs:57
    }
    // sequential fp64 sum in index order (Sampler.cs:58)
    double s1 = 0.0;
    {
        const int n0 = S < 32 ? S : 32;
        for (int j = 0; j < n0; ++j) s1 = __dadd_rn(s1, shfl_d(p[0], j));
        for (int j = 32; j < S; ++j) s1 = __dadd_rn(s1, shfl_d(p[1], j - 32));
    }
#pragma unroll
    for (int s = 0; s < 2; ++s) p[s] = __ddiv_rn(p[s], s1);   // :60 (0 / s1 = 0 on padding)

    if (o.top_p < 1.0f) {   // Sampler.cs:62-75
        const double thr = static_cast<double>(__fsub_rn(1.0f, o.top_p));
        uint64_t pk[2];
        uint32_t tag[2];
#pragma unroll
        for (int s = 0; s < 2; ++s) {
            const int e = s * 32 + lane;
            pk[s] = e < S ? static_cast<uint64_t>(__double_as_longlong(p[s])) : ~0ull;
            tag[s] = static_cast<uint32_t>(e);   // index-order position; the order of positions is the index order
        }
        warp_sort_pair<2>(pk, tag, lane);
        double cum = 0.0;
        int m = S - 1;
        {
            const int n0 = (S - 1) < 32 ? (S - 1) : 32;
            bool done = false;
            for (int j = 0; j < n0; ++j) {
                cum = __dadd_rn(cum, __longlong_as_double(static_cast<long long>(shfl_u64(pk[0], j))));
                if (!(cum <= thr)) {
                    m = j;
                    done = true;
                    break;
                }
            }
            if (!done)
                for (int j = 32; j < S - 1; ++j) {
                    cum = __dadd_rn(cum, __longlong_as_double(static_cast<long long>(shfl_u64(pk[1], j - 32))));
                    if (!(cum <= thr)) {
                        m = j;
                        break;
                    }
                }
        }
#pragma unroll
        for (int s = 0; s < 2; ++s) {
            const int j = s * 32 + lane;
            if (j < S) misc.flags[tag[s]] = j < m ? 1 : 0;
        }
        __syncwarp();
#pragma unroll
        for (int s = 0; s < 2; ++s) {
            const int e = s * 32 + lane;
            if (e < S && misc.flags[e]) p[s] = 0.0;
        }
        __syncwarp();
        double s2 = 0.0;   // probs.Sum() (:73)
        {
            const int n0 = S < 32 ? S : 32;
            for (int j = 0; j < n0; ++j) s2 = __dadd_rn(s2, shfl_d(p[0], j));
            for (int j = 32; j < S; ++j) s2 = __dadd_rn(s2, shfl_d(p[1], j - 32));
        }
#pragma unroll
        for (int s = 0; s < 2; ++s) p[s] = __ddiv_rn(p[s], s2);   // :74
    }
    // inverse-CDF draw (Sampler.cs:77-87)
    double acc = 0.0;
    int last = 0, res = -1;
    {
        const int n0 = S < 32 ? S : 32;
        for (int j = 0; j < n0 && res < 0; ++j) {
            const double v = shfl_d(p[0], j);
            const int id = __shfl_sync(kFull, idx[0], j);
            if (v <= 0.0) continue;
            acc = __dadd_rn(acc, v);
            last = id;
            if (r < acc) res = id;
        }
        for (int j = 32; j < S && res < 0; ++j) {
            const double v = shfl_d(p[1], j - 32);
            const int id = __shfl_sync(kFull, idx[1], j - 32);
            if (v <= 0.0) continue;
            acc = __dadd_rn(acc, v);
            last = id;
            if (r < acc) res = id;
        }
    }
    if (out_probs) {
#pragma unroll
        for (int s = 0; s < 2; ++s)
            if (s * 32 + lane < S) out_probs[idx[s]] = p[s];
    }
    return res < 0 ? last : res;
}

// ---------------------------------------------------------------- the kernel
template <int VW>
__device__ __forceinline__ void process_vectors(const unsigned char* sl, int nvec, int lo_al, int hi_al,
                                                const RowCtx& c, int tid, float (&x)[kRegElems],
                                                float& tmax, float& bestv, int& besti) {
    constexpr int G = kRegElems / VW;
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const int qv = tid + g * kThreads;
        if (qv < nvec) {
            float v[VW];
            load_vec<VW>(sl, qv, v);
            const int q0 = qv * VW;
            const int i0 = q0 < lo_al ? q0 : q0 - lo_al + hi_al;
            const uint32_t bits = c.pen_on ? c.bitmap[i0 >> 5] : 0u;
#pragma unroll
            for (int e = 0; e < VW; ++e) {
                const float t = transform(v[e], i0 + e, bits, c);
                x[g * VW + e] = t;
                tmax = fmaxf(tmax, t);
                if (t > bestv) {
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

__global__ void __launch_bounds__(kThreads + 32) sampler_kernel(const __grid_constant__ LaunchParams p) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int S_ = p.n_stages;
    const int stage_bytes = kMetaBytes + kKeepBytes + p.stage_logit_bytes + p.stage_hist_cap * 4;
    unsigned char* stages = smem;
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(S_) * stage_bytes);
    uint64_t* empty_bar = full_bar + S_;
    uint32_t* bitmap = reinterpret_cast<uint32_t*>(empty_bar + S_);
    Cand* cand = reinterpret_cast<Cand*>(bitmap + ((p.bitmap_words + 1) & ~1));
    SmemMisc& misc = *reinterpret_cast<SmemMisc*>(cand + kCandCap);

    const int first = blockIdx.x;
    const int gstride = gridDim.x;
    const int n_my = first < p.total_rows ? (p.total_rows - 1 - first) / gstride + 1 : 0;

    if (tid == 0) {
        for (int s = 0; s < S_; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        fence_mbar_init();
        misc.cand_count = 0;
        misc.issued = 0;
    }
    for (int i = tid; i < p.bitmap_words; i += blockDim.x) bitmap[i] = 0u;
    __syncthreads();

    if (warp == kWarps) {
        // ================= producer warp: plans rows and issues the bulk copies =================
        bool alive = true;
        for (int k0 = 0; k0 < n_my && alive; k0 += 32) {
            // lane j prefetches the metadata of the CTA's row k0 + j
            const int kj = k0 + lane;
            RowMeta m;
            const DevSegment* sg = &p.seg[0];
            const unsigned char* row_ptr = nullptr;
            int esize = 4;
            uint32_t bytes = 0;
            if (kj < n_my) {
                const int r = first + kj * gstride;
                int s = 0;
                for (int i = 1; i < p.n_segs; ++i)
                    if (r >= p.seg[i].row_begin) s = i;
                sg = &p.seg[s];
                const int local = r - sg->row_begin;
                const int opt_raw = sg->opt_index ? sg->opt_index[local] : 0;
                m.row = r;
                m.seg = s;
                m.local = local;
                m.step = sg->steps ? sg->steps[local] : 0x7fffffff;
                m.uniform = sg->uniforms ? sg->uniforms[local] : 0.0;
                int64_t hb = 0, he = 0;
                if (sg->kind == 0 && sg->hist_offsets) {
                    hb = sg->hist_offsets[local];
                    he = sg->hist_offsets[local + 1];
                }
                m.opt_ok = (opt_raw >= 0 && opt_raw < p.n_opts) ? 1 : 0;
                if (m.opt_ok) {
                    m.opt = p.n_opts <= kInlineOptions ? p.inl_opts[opt_raw] : p.dev_opts[opt_raw];
                } else {
                    m.opt = DevOptions{0, 0, 1.0f, 1.0f, 1.0f};
                }
                const int V = sg->vocab;
                esize = sg->dtype == 0 ? 4 : 2;
                const int VWe = 16 / esize;
                m.pen_on = (m.opt_ok && sg->kind == 0 && m.opt.rep_penalty != 1.0f && he > hb) ? 1 : 0;
                m.hist_begin = hb;
                m.hist_len = static_cast<int32_t>(he - hb);
                m.lo_al = V;
                m.hi_al = V;
                if (sg->kind == 0 && sg->sup_lo < sg->sup_hi) {
                    const int la = (sg->sup_lo + VWe - 1) / VWe * VWe;
                    const int ha = sg->sup_hi / VWe * VWe;
                    if (la < ha) {
                        m.lo_al = la;
                        m.hi_al = ha;
                    }
                }
                m.keep = (sg->kind == 0 && sg->eos >= m.lo_al && sg->eos < m.hi_al && m.step >= sg->min_new) ? 1 : 0;
                m.direct = sg->bulk_ok ? 0 : 1;
                m.hs_lo = 0;
                m.hs_hi = 0;
                if (m.pen_on && sg->hist_aligned && p.stage_hist_cap > 0) {
                    int64_t a = (hb + 3) / 4 * 4;
                    int64_t b = he / 4 * 4;
                    if (b > a + p.stage_hist_cap) b = a + p.stage_hist_cap;
                    if (b > a) {
                        m.hs_lo = static_cast<int32_t>(a - hb);
                        m.hs_hi = static_cast<int32_t>(b - hb);
                    }
                }
                row_ptr = static_cast<const unsigned char*>(sg->logits) +
                          static_cast<int64_t>(local) * sg->row_stride * esize;
                if (!m.direct) bytes += static_cast<uint32_t>((m.lo_al + V - m.hi_al) * esize) + (m.keep ? 16u : 0u);
                bytes += static_cast<uint32_t>(m.hs_hi - m.hs_lo) * 4u;
            }
            const int nb = (n_my - k0) < 32 ? (n_my - k0) : 32;
            for (int j = 0; j < nb; ++j) {
                bool ok = true;
                if (lane == j) {
                    const int k = k0 + j;
                    const int s = k % S_;
                    const int n = k / S_;
                    if (n > 0) ok = mbar_wait_bounded(&empty_bar[s], static_cast<uint32_t>((n - 1) & 1));
                    if (ok) {
                        unsigned char* st = stages + static_cast<size_t>(s) * stage_bytes;
                        *reinterpret_cast<RowMeta*>(st) = m;
                        unsigned char* keep_dst = st + kMetaBytes;
                        unsigned char* log_dst = keep_dst + kKeepBytes;
                        unsigned char* hist_dst = log_dst + p.stage_logit_bytes;
                        fence_proxy_async();
                        mbar_arrive_expect_tx(&full_bar[s], bytes);
                        if (!m.direct) {
                            const int V = sg->vocab;
                            if (m.lo_al > 0) bulk_g2s(log_dst, row_ptr, static_cast<uint32_t>(m.lo_al * esize), &full_bar[s]);
                            if (V > m.hi_al)
                                bulk_g2s(log_dst + m.lo_al * esize, row_ptr + static_cast<int64_t>(m.hi_al) * esize,
                                         static_cast<uint32_t>((V - m.hi_al) * esize), &full_bar[s]);
                            if (m.keep) {
                                const int VWe = 16 / esize;
                                bulk_g2s(keep_dst, row_ptr + static_cast<int64_t>(sg->eos / VWe * VWe) * esize, 16u,
                                         &full_bar[s]);
                            }
                        }
                        if (m.hs_hi > m.hs_lo)
                            bulk_g2s(hist_dst, sg->hist_ids + m.hist_begin + m.hs_lo,
                                     static_cast<uint32_t>(m.hs_hi - m.hs_lo) * 4u, &full_bar[s]);
                        misc.issued = k + 1;
                    } else {
                        atomicOr(p.err, kErrTimeout);
                    }
                }
                ok = __shfl_sync(kFull, ok ? 1 : 0, j) != 0;
                if (!ok) {
                    alive = false;
                    break;
                }
            }
        }
        return;
    }

    // ================= compute warps =================
    for (int k = 0; k < n_my; ++k) {
        const int s = k % S_;
        unsigned char* st = stages + static_cast<size_t>(s) * stage_bytes;
        const bool ok = mbar_wait_bounded(&full_bar[s], static_cast<uint32_t>((k / S_) & 1));
        if (cbar_or(!ok)) {
            if (tid == 0) atomicOr(p.err, kErrTimeout);
            // drain: wait (bounded) for every copy the producer issued after this row
            if (tid == 0) {
                const int issued = *reinterpret_cast<volatile int*>(&misc.issued);
                for (int kk = k; kk < issued; ++kk) mbar_wait_bounded(&full_bar[kk % S_], static_cast<uint32_t>((kk / S_) & 1));
            }
            cbar();
            return;
        }
        const RowMeta m = *reinterpret_cast<const RowMeta*>(st);
        const DevSegment& g = p.seg[m.seg];
        const unsigned char* keep_src = st + kMetaBytes;
        unsigned char* sl = st + kMetaBytes + kKeepBytes;
        const int32_t* sh = reinterpret_cast<const int32_t*>(sl + p.stage_logit_bytes);
        const int V = g.vocab;
        const int dtype = g.dtype;
        const int VWe = dtype == 0 ? 4 : 8;
        const int NA = m.lo_al + (V - m.hi_al);
        const int nvec = (NA + VWe - 1) / VWe;   // bulk-copied rows have NA % VWe == 0
        double* out_probs = g.out_probs ? g.out_probs + static_cast<int64_t>(m.local) * V : nullptr;

        if (!m.opt_ok) {
            if (tid == 0) {
                atomicOr(p.err, kErrBadOption);
                g.out_ids[m.local] = -1;
            }
            cbar();
            if (tid == 0) mbar_arrive(&empty_bar[s]);
            continue;
        }
        const DevOptions o = m.opt;

        // ---- unaligned rows: the compute warps stage the active ids themselves
        if (m.direct) {
            const unsigned char* row = static_cast<const unsigned char*>(g.logits) +
                                       static_cast<int64_t>(m.local) * g.row_stride * (dtype == 0 ? 4 : 2);
            for (int q = tid; q < nvec * VWe; q += kThreads) {
                const int i = q < m.lo_al ? q : q - m.lo_al + m.hi_al;
                if (dtype == 0)
                    reinterpret_cast<float*>(sl)[q] = i < V ? reinterpret_cast<const float*>(row)[i] : neg_inf();
                else   // padding past V reads as bf16 -inf
                    reinterpret_cast<uint16_t*>(sl)[q] = i < V ? reinterpret_cast<const uint16_t*>(row)[i] : 0xff80u;
            }
        }

        // ---- repetition-penalty bitmap: Distinct() over the history (Sampler.cs:28)
        bool bad = false;
        if (m.pen_on) {
            const int32_t* gh = g.hist_ids + m.hist_begin;
            const int nst = m.hs_hi - m.hs_lo;
            for (int c4 = tid; c4 < nst / 4; c4 += kThreads) {
                const int4 v = reinterpret_cast<const int4*>(sh)[c4];
                const int ids[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if (static_cast<unsigned>(ids[j]) >= static_cast<unsigned>(V)) {
                        bad = true;
                    } else {
                        atomicOr(&bitmap[ids[j] >> 5], 1u << (ids[j] & 31));
                    }
                }
            }
            const int rest = m.hist_len - nst;   // ids outside the staged span: [0, hs_lo) and [hs_hi, len)
            for (int q = tid; q < rest; q += kThreads) {
                const int i = q < m.hs_lo ? q : q - m.hs_lo + m.hs_hi;
                const int id = gh[i];
                if (static_cast<unsigned>(id) >= static_cast<unsigned>(V)) {
                    bad = true;
                } else {
                    atomicOr(&bitmap[id >> 5], 1u << (id & 31));
                }
            }
            if (bad) atomicOr(p.err, kErrHistRange);
        }
        if (m.pen_on || m.direct) cbar();

        RowCtx c;
        c.vocab = V;
        c.kind = g.kind;
        c.sup_lo = g.sup_lo;
        c.sup_hi = g.sup_hi;
        c.eos = g.eos;
        c.eos_blocked = m.step < g.min_new;
        c.pen_on = m.pen_on != 0;
        c.pen = o.rep_penalty;
        c.pen_rcp = __drcp_rn(static_cast<double>(o.rep_penalty));
        c.sample = o.do_sample != 0;
        c.inv_t = __fdiv_rn(1.0f, o.temperature);
        c.bitmap = bitmap;

        const bool big = nvec > kThreads * (kRegElems / VWe);
        float x[kRegElems];
        float tmax = neg_inf();
        float bestv = neg_inf();
        int besti = 0x7fffffff;
        float xk = neg_inf();   // EOS when staged separately (thread 0)
        if (!big) {
            if (dtype == 0)
                process_vectors<4>(sl, nvec, m.lo_al, m.hi_al, c, tid, x, tmax, bestv, besti);
            else
                process_vectors<8>(sl, nvec, m.lo_al, m.hi_al, c, tid, x, tmax, bestv, besti);
        }
        if (m.keep && tid == 0) {
            float v;
            if (m.direct) {
                const unsigned char* row = static_cast<const unsigned char*>(g.logits) +
                                           static_cast<int64_t>(m.local) * g.row_stride * (dtype == 0 ? 4 : 2);
                v = load_elem(row, g.eos, dtype);
            } else {
                v = load_elem(keep_src, g.eos % VWe, dtype);
            }
            const uint32_t bits = c.pen_on ? bitmap[g.eos >> 5] : 0u;
            xk = transform(v, g.eos, bits, c);
            tmax = fmaxf(tmax, xk);
            if (xk > bestv || (xk == bestv && g.eos < besti)) {
                bestv = xk;
                besti = g.eos;
            }
        }

        int result = -1;
        bool general = false;
        if (big) {
            general = true;   // handled below, after the stage is copied out
        } else if (!c.sample) {
            // ---- greedy (Sampler.cs:37, 90-95): first index of the maximum
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
                misc.red_v[warp] = bestv;
                misc.red_i[warp] = besti;
            }
            cbar();
            if (tid == 0) {
                float bv = misc.red_v[0];
                int bi = misc.red_i[0];
                for (int w = 1; w < kWarps; ++w)
                    if (misc.red_v[w] > bv || (misc.red_v[w] == bv && misc.red_i[w] < bi)) {
                        bv = misc.red_v[w];
                        bi = misc.red_i[w];
                    }
                // all -inf: the reference's scan never moves off index 0
                g.out_ids[m.local] = is_neg_inf(bv) ? 0 : bi;
                mbar_arrive(&empty_bar[s]);
            }
            if (out_probs)
                for (int i = tid; i < V; i += kThreads) out_probs[i] = 0.0;
            if (m.pen_on)
                for (int i = tid; i < p.bitmap_words; i += kThreads) bitmap[i] = 0u;
            cbar();
            continue;
        } else {
            const int K = o.top_k;
            const bool small_ok = K > 0 && K < V && K <= kSmallK;
            float tau = neg_inf();
            if (small_ok) {
                // tau_w = ceil(K/4)-th largest lane maximum of this warp
                const int cw = (K + kWarps - 1) / kWarps;
                uint64_t lk[1] = {static_cast<uint64_t>(~okey(tmax))};
                warp_sort<1>(lk, lane);
                const float tw = okey_inv(~static_cast<uint32_t>(__shfl_sync(kFull, lk[0], cw - 1)));
                if (lane == 0) misc.tau_w[warp] = tw;
            }
            if (out_probs)
                for (int i = tid; i < V; i += kThreads) out_probs[i] = 0.0;
            cbar();   // tau_w visible; the stage has been read: hand it back to the producer
            if (tid == 0) mbar_arrive(&empty_bar[s]);
            if (m.pen_on)
                for (int i = tid; i < p.bitmap_words; i += kThreads) bitmap[i] = 0u;
            if (small_ok) {
                tau = misc.tau_w[0];
#pragma unroll
                for (int w = 1; w < kWarps; ++w) tau = fminf(tau, misc.tau_w[w]);
            }
            if (!small_ok || is_neg_inf(tau)) {
                general = true;
            } else {
                // ---- candidates x >= tau -> shared buffer (warp-scan positions, one atomic per warp)
                int cnt = 0;
#pragma unroll
                for (int e = 0; e < kRegElems; ++e) cnt += (x[e] >= tau) ? 1 : 0;
                if (tid == 0 && m.keep && xk >= tau) ++cnt;
                int incl = cnt;
#pragma unroll
                for (int off = 1; off < 32; off <<= 1) {
                    const int y = __shfl_up_sync(kFull, incl, off);
                    if (lane >= off) incl += y;
                }
                uint32_t base = 0;
                if (lane == 31) base = atomicAdd(&misc.cand_count, static_cast<uint32_t>(incl));
                base = __shfl_sync(kFull, base, 31);
                int pos = static_cast<int>(base) + incl - cnt;
                if (cnt > 0) {
                    const int VWl = VWe;
#pragma unroll
                    for (int e = 0; e < kRegElems; ++e) {
                        if (x[e] >= tau) {
                            if (pos < kCandCap) {
                                const int gg = e / VWl;
                                const int qv = tid + gg * kThreads;
                                const int q = qv * VWl + (e - gg * VWl);
                                const int i = q < m.lo_al ? q : q - m.lo_al + m.hi_al;
                                cand[pos] = Cand{x[e], i};
                            }
                            ++pos;
                        }
                    }
                    if (tid == 0 && m.keep && xk >= tau) {
                        if (pos < kCandCap) cand[pos] = Cand{xk, g.eos};
                        ++pos;
                    }
                }
                cbar();
                if (warp == 0) {
                    const int C = static_cast<int>(misc.cand_count);
                    int res = -1;
                    if (C <= kCandCap) res = small_path(cand, C, o, m.uniform, out_probs, misc, lane);
                    if (lane == 0) {
                        misc.decision = res;
                        if (res >= 0) g.out_ids[m.local] = res;
                        misc.cand_count = 0;
                    }
                }
                cbar();
                result = misc.decision;
                general = result < 0;
            }
        }

        if (general) {
            // ================= general path over per-CTA global scratch =================
            char* gbase = p.gscratch + static_cast<int64_t>(blockIdx.x) * p.gscratch_stride;
            const int vpad = (p.vmax + 31) & ~31;
            float* gx = reinterpret_cast<float*>(gbase);
            double* gp = reinterpret_cast<double*>(gbase + static_cast<int64_t>(vpad) * 4);
            uint4* gs = reinterpret_cast<uint4*>(gbase + static_cast<int64_t>(vpad) * 12);
            int sort_n = 1;
            while (sort_n < V) sort_n <<= 1;
            for (int i = tid; i < V; i += kThreads) gx[i] = neg_inf();
            cbar();
            if (!big) {
                const int G = kRegElems / VWe;
                for (int gg = 0; gg < G; ++gg) {
                    const int qv = tid + gg * kThreads;
                    if (qv < nvec) {
                        for (int e = 0; e < VWe; ++e) {
                            const int q = qv * VWe + e;
                            const int i = q < m.lo_al ? q : q - m.lo_al + m.hi_al;
                            if (i < V) gx[i] = x[gg * VWe + e];
                        }
                    }
                }
            } else {
                // rows with more than 3072 active ids: transform straight from the stage
                for (int qv = tid; qv < nvec; qv += kThreads) {
                    const int q0 = qv * VWe;
                    const int i0 = q0 < m.lo_al ? q0 : q0 - m.lo_al + m.hi_al;
                    const uint32_t bits = c.pen_on ? bitmap[i0 >> 5] : 0u;
                    for (int e = 0; e < VWe && i0 + e < V; ++e) {
                        const float t = transform(load_elem(sl, q0 + e, dtype), i0 + e, bits, c);
                        gx[i0 + e] = t;
                        tmax = fmaxf(tmax, t);
                        if (t > bestv) {
                            bestv = t;
                            besti = i0 + e;
                        }
                    }
                }
            }
            if (tid == 0 && m.keep) gx[g.eos] = xk;
            if (big) {
                if (out_probs)
                    for (int i = tid; i < V; i += kThreads) out_probs[i] = 0.0;
                cbar();
                if (tid == 0) mbar_arrive(&empty_bar[s]);
                if (m.pen_on)
                    for (int i = tid; i < p.bitmap_words; i += kThreads) bitmap[i] = 0u;
            }
            cbar();
            if (big && !c.sample) {
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
                    misc.red_v[warp] = bestv;
                    misc.red_i[warp] = besti;
                }
                cbar();
                if (tid == 0) {
                    float bv = misc.red_v[0];
                    int bi = misc.red_i[0];
                    for (int w = 1; w < kWarps; ++w)
                        if (misc.red_v[w] > bv || (misc.red_v[w] == bv && misc.red_i[w] < bi)) {
                            bv = misc.red_v[w];
                            bi = misc.red_i[w];
                        }
                    g.out_ids[m.local] = is_neg_inf(bv) ? 0 : bi;
                }
                cbar();
                continue;
            }
            const float mx = block_max(tmax, misc, lane, warp);
            cbar();
            const int res = general_path(c, o, m.uniform, mx, gx, gp, gs, sort_n, out_probs, misc, tid);
            if (tid == 0) g.out_ids[m.local] = res;
        }
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

}  // namespace

// ---------------------------------------------------------------- host-side launch helpers
size_t sampler_smem_bytes(const LaunchParams& p) {
    const size_t stage = kMetaBytes + kKeepBytes + static_cast<size_t>(p.stage_logit_bytes) +
                         static_cast<size_t>(p.stage_hist_cap) * 4;
    size_t b = stage * p.n_stages;
    b += 2 * sizeof(uint64_t) * p.n_stages;
    b += sizeof(uint32_t) * ((p.bitmap_words + 1) & ~1);
    b += sizeof(Cand) * kCandCap;
    b += sizeof(SmemMisc);
    return b;
}

int64_t sampler_gscratch_stride(int vmax) {
    const int64_t vpad = (vmax + 31) & ~31;
    int64_t sort_n = 1;
    while (sort_n < vmax) sort_n <<= 1;
    int64_t b = vpad * 4 + vpad * 8 + sort_n * 16;
    return (b + 255) & ~static_cast<int64_t>(255);
}

int sampler_ctas_per_sm(size_t smem) {
    static size_t configured = 0;
    if (smem > 48 * 1024 && smem > configured) {
        if (cudaFuncSetAttribute(sampler_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem)) != cudaSuccess)
            return 0;
        configured = smem;
    }
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, sampler_kernel, kThreads + 32, smem) != cudaSuccess)
        return 0;
    return n;
}

cudaError_t launch_sampler(const LaunchParams& p, int grid, size_t smem, cudaStream_t stream) {
    sampler_kernel<<<grid, kThreads + 32, smem, stream>>>(p);
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
