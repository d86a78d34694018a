// vw_rowwarp.cuh -- the warp-per-row candidate kernel.  Included by vw_sampler.cu inside its namespace; uses that
// file's helpers (okey, softmax_num, penalize, transform, replay_candidates, ...).
//
// One warp per row and no block barrier: warp g of the grid takes rows g, g + G, g + 2G, ... (G = warps launched),
// so the warps of a CTA never wait for one another.  A row is read with 16-byte vector loads straight from
// global memory (the skipped suppress span is never read).  Per sampling row with 0 < K <= 64:
//   1. history ids -> a bitmap of the ids (Distinct(), Sampler.cs:28);
//   2. mark pass: lane l reads vectors l, l + 32, ... of each part (every warp load is 512 contiguous bytes); a
//      vector is marked when its largest raw value is >= x0, the smallest raw value whose temperature-scaled value
//      reaches the threshold tau (a penalty > 1 only lowers values, so raw >= x0 is necessary for a candidate);
//      vectors holding suppressed ids or EOS are always marked;
//   3. the marked vectors are listed in index order (one ballot per step of 32 vectors) and re-read (L1 / L2); each
//      element with raw >= x0 becomes a raw candidate, and each raw candidate's exact value (penalty, mask,
//      temperature: Sampler.cs:31, TalkerGenerator.cs:247-248, Sampler.cs:40) is kept when >= tau: the candidates,
//      in index order (lane l holds positions l, l + 32, ... from here on);
//   4. with K <= C <= 256 candidates the K-th largest value is >= tau, so the candidates hold every survivor of the
//      top-k cut (Sampler.cs:42-49); a count over value buckets finds the K-th largest;
//   5. softmax numerators (libm exp, Sampler.cs:57) in 64-bit fixed point, the top-p cut over the ascending order
//      (Sampler.cs:62-72) and the inverse-CDF draw over index order (Sampler.cs:77-87), each decision certified
//      against the error band of the parallel sums, else the warp replays the row in the reference's order.
// A threshold that misses (C outside [K, 256]) is rebuilt from the row's own values, except that one a few
// candidates short is first lowered along the tail its candidates show; rows the kernel does not take
// (top-k off or > 64, a penalty < 1, unaligned rows, too many candidates) go to the whole-row kernel.

constexpr int kRwWarps = 4;       // warps per CTA, each on its own rows
constexpr int kRwBatch = 8;       // 16-byte vectors per lane in flight per load batch
constexpr int kRwPre = 4;         // re-read vectors per lane in flight (marked vectors, 32 per step)
constexpr int kRwHistBatch = 8;   // 16-byte history loads per lane in flight
constexpr int kRwCandCap = 256;   // candidates (exact value >= tau) per row
constexpr int kRwSlots = kRwCandCap / 32;
constexpr int kRwRawCap = 384;    // raw candidates (raw value >= x0) per row

// Per-warp shared memory.
struct __align__(16) RwArea {
    unsigned long long key[kRwCandCap]; // candidates in index order: okey(t) << 32 | id
    union __align__(16) {
        struct {
            float v[kRwRawCap];          // raw candidates (raw value, id), index order
            int32_t id[kRwRawCap];
        } raw;
        struct {
            unsigned long long sv[64];   // survivors in index order (key as in `key`)
            double e[64];                // their softmax numerators
            unsigned long long f[64];    // the same in fixed point, round(e * 2^52)
            uint32_t sk[64];             // survivors in ascending (value, index) order: (value - kth) << 6 | d
            int32_t kept[64];            // survivor d kept by top-p
            uint32_t blist[kRwCandCap];  // the values of the K-th largest's bucket
        } sel;
        int32_t rflags[kCandCap];        // replay scratch
    } u;
    uint16_t vlist[kRwRawCap];          // marked vectors (global vector index), index order
    int32_t bcount[kRankBuckets];
};
static_assert(sizeof(RwArea) % 16 == 0, "RwArea alignment");

__device__ __forceinline__ float prev_float(float x) {   // the next float toward -inf (x finite)
    const uint32_t u = __float_as_uint(x);
    if ((u & 0x7fffffffu) == 0) return -__uint_as_float(1u);
    return __uint_as_float((u & 0x80000000u) ? u + 1u : u - 1u);
}

// The smallest raw value whose scaled value fl(x * c) can reach tau, minus a margin: fl(x * c) is monotone in x, and
// fl(tau / c) is within two ulps of the true boundary, so three steps down is a lower bound.
__device__ __forceinline__ float raw_threshold(float tau, float c) {
    float y = __fdiv_rn(tau, c);
    if (!(fabsf(y) < pos_inf())) return y;   // +-inf / nan: handled by the caller (no candidates)
    y = prev_float(prev_float(prev_float(y)));
    return y;
}

template <int VW>
__device__ __forceinline__ float vec_max(const uint4& u);
template <>
__device__ __forceinline__ float vec_max<4>(const uint4& u) {
    return fmaxf(fmaxf(__uint_as_float(u.x), __uint_as_float(u.y)), fmaxf(__uint_as_float(u.z), __uint_as_float(u.w)));
}
template <>
__device__ __forceinline__ float vec_max<8>(const uint4& u) {   // bf16 pairs: the larger of each pair, widened
    auto mx2 = [](uint32_t a) { return fmaxf(__uint_as_float(a << 16), __uint_as_float(a & 0xffff0000u)); };
    return fmaxf(fmaxf(mx2(u.x), mx2(u.y)), fmaxf(mx2(u.z), mx2(u.w)));
}
template <int VW>
__device__ __forceinline__ float vec_elem(const uint4& u, int e) {   // element e (compile-time after unrolling)
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    if (VW == 4) return __uint_as_float(w[e]);
    return __uint_as_float((e & 1) ? (w[e >> 1] & 0xffff0000u) : (w[e >> 1] << 16));   // Bf16.ToFloat
}
__device__ __forceinline__ uint4 neg_inf_vec(int VW) {
    const uint32_t n = VW == 4 ? 0xff800000u : 0xff80ff80u;
    return make_uint4(n, n, n, n);
}

// Mark pass over one part (global vectors [v0, v0 + nv), lane l taking vectors l, l + 32, ...: each warp load is 512
// contiguous bytes): bit i of the result is set when vector v0 + 32 i + l holds a raw value >= x0, or holds
// suppressed ids ([spec_a, spec_b]) or the blocked EOS (ev).
template <int VW>
__device__ __forceinline__ uint32_t mark_part(const uint4* row, int v0, int nv, float x0, int spec_a, int spec_b, int ev,
                                              int lane) {
    uint32_t marks = 0u;
    const int steps = (nv + 31) >> 5;
    for (int b0 = 0; b0 < steps; b0 += kRwBatch) {
        uint4 v[kRwBatch];
#pragma unroll
        for (int i = 0; i < kRwBatch; ++i) {
            const int q = ((b0 + i) << 5) + lane;
            v[i] = q < nv ? __ldg(row + v0 + q) : neg_inf_vec(VW);
        }
        uint32_t m = 0u;
#pragma unroll
        for (int i = 0; i < kRwBatch; ++i) {
            const int q = ((b0 + i) << 5) + lane, gv = v0 + q;
            const bool spec = q < nv && ((gv >= spec_a && gv <= spec_b) || gv == ev);
            if (spec || vec_max<VW>(v[i]) >= x0) m |= 1u << i;
        }
        marks |= m << b0;
    }
    return marks;
}

// Lists the marked vectors of one part (bit i of lane l: vector v0 + 32 i + l) in index order at a.vlist[o..].
__device__ __forceinline__ void list_part(uint32_t marks, int v0, int nv, uint16_t* vlist, int o, int lane) {
    const int steps = (nv + 31) >> 5;
    const uint32_t lt = (1u << lane) - 1u;
    for (int i = 0; i < steps; ++i) {
        const bool on = (marks >> i) & 1u;
        const unsigned bal = __ballot_sync(kFull, on);
        if (on) vlist[o + __popc(bal & lt)] = static_cast<uint16_t>(v0 + (i << 5) + lane);
        o += __popc(bal);
    }
}

// Exclusive prefix of v over the lanes; `total` = the sum over all lanes.
__device__ __forceinline__ int warp_excl_i(int v, int lane, int& total) {
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(kFull, incl, o);
        if (lane >= o) incl += y;
    }
    total = __shfl_sync(kFull, incl, 31);
    return incl - v;
}
__device__ __forceinline__ unsigned long long warp_incl_ull(unsigned long long v, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long y = __shfl_up_sync(kFull, v, o);
        if (lane >= o) v += y;
    }
    return v;
}

// What the warp kernel needs about one row.
struct RwRow {
    const uint4* row;        // the row's vectors
    double uniform, pen_rcp;
    float inv_t, pen;
    int row_id, seg, opt, local;
    int V, kind, sup_lo, sup_hi, eos;
    bool eos_blocked, pen_on;
    const int32_t* hist;     // the row's history ids (pen_on)
    int hlen;
};

__device__ __forceinline__ bool bm_test(const uint32_t* bm, int id) { return (bm[id >> 5] >> (id & 31)) & 1u; }

// The exact value of one element: repetition penalty (Sampler.cs:31) -> suppress mask (TalkerGenerator.cs:247-248)
// -> temperature (Sampler.cs:40).
__device__ __forceinline__ float rw_exact(float raw, int id, const uint32_t* bm, const RwRow& r) {
    float v = raw;
    if (r.pen_on && bm_test(bm, id)) v = penalize(v, r.pen, r.pen_rcp);
    if (r.kind == 0 && ((id >= r.sup_lo && id < r.sup_hi && id != r.eos) || (id == r.eos && r.eos_blocked)))
        v = neg_inf();
    return __fmul_rn(v, r.inv_t);
}
// The same without temperature (greedy rows: Sampler.cs:37 takes the argmax of the penalised, masked row).
__device__ __forceinline__ float rw_exact_greedy(float raw, int id, const uint32_t* bm, const RwRow& r) {
    float v = raw;
    if (r.pen_on && bm_test(bm, id)) v = penalize(v, r.pen, r.pen_rcp);
    if (r.kind == 0 && ((id >= r.sup_lo && id < r.sup_hi && id != r.eos) || (id == r.eos && r.eos_blocked)))
        v = neg_inf();
    return v;
}

// History ids -> bitmap bm (cleared first; id V is the sink of out-of-range ids).  Returns true when an id was
// outside [0, V) (the reference throws there, Sampler.cs:30).
__device__ bool rw_history(const int32_t* hist, int len, int V, uint32_t* bm, int lane) {
    const int words = (V >> 5) + 1;
    for (int w = lane; w < words; w += 32) bm[w] = 0u;
    __syncwarp();
    bool bad = false;
    auto put = [&](int id) {
        const unsigned u = static_cast<unsigned>(id);
        bad |= u >= static_cast<unsigned>(V);
        const int k = u < static_cast<unsigned>(V) ? id : V;
        atomicOr(&bm[k >> 5], 1u << (k & 31));
    };
    // ragged head up to a 16-byte boundary, then four ids per 16-byte load, then the tail
    const int head = min(len, static_cast<int>((16u - (reinterpret_cast<uintptr_t>(hist) & 15u)) & 15u) >> 2);
    if (lane < head) put(hist[lane]);
    const int4* h4 = reinterpret_cast<const int4*>(hist + head);
    const int n4 = (len - head) >> 2;
    for (int j0 = 0; j0 < n4; j0 += kRwHistBatch * 32) {
        int4 w[kRwHistBatch];
#pragma unroll
        for (int k = 0; k < kRwHistBatch; ++k) {
            const int j = j0 + k * 32 + lane;
            w[k] = j < n4 ? __ldg(h4 + j) : make_int4(0, 0, 0, 0);
        }
#pragma unroll
        for (int k = 0; k < kRwHistBatch; ++k) {
            if (j0 + k * 32 + lane >= n4) continue;
            put(w[k].x);
            put(w[k].y);
            put(w[k].z);
            put(w[k].w);
        }
    }
    const int t0 = head + 4 * n4;
    if (lane < len - t0) put(hist[t0 + lane]);
    __syncwarp();
    return __any_sync(kFull, bad);
}

// Steps 2-3 for one threshold: candidates (index order) into a.key, their number in C, the largest value in mx.
// Returns false when the list overflows (too many marked vectors or raw candidates: the threshold is too low).
template <int VW>
__device__ bool rw_collect(const RwRow& r, const DevSegment& sg, float tau, float x0, uint32_t* bm, bool& bm_ready,
                           bool& hist_bad, RwArea& a, int lane, int& C, float& mx) {
    constexpr int vsh = VW == 4 ? 2 : 3;
    // marks, with the vectors holding suppressed ids (and EOS while it is blocked) always marked
    const int ev = (r.kind == 0 && r.eos_blocked && r.eos >= 0 && r.eos < r.V) ? (r.eos >> vsh) : -1;
    const uint32_t mA = mark_part<VW>(r.row, 0, sg.va, x0, sg.spec_a, sg.spec_b, ev, lane);
    const uint32_t mC = sg.vc > 0 ? mark_part<VW>(r.row, sg.c0, sg.vc, x0, sg.spec_a, sg.spec_b, ev, lane) : 0u;
    // list in index order: part A, the EOS vector, part C
    const int tA = __reduce_add_sync(kFull, __popc(mA)), tC = __reduce_add_sync(kFull, __popc(mC));
    const int ne = sg.eosv >= 0 ? 1 : 0;
    const int M = tA + ne + tC;
    if (M > kRwRawCap) return false;
    list_part(mA, 0, sg.va, a.vlist, 0, lane);
    if (ne && lane == 0) a.vlist[tA] = static_cast<uint16_t>(sg.eosv);
    if (sg.vc > 0) list_part(mC, sg.c0, sg.vc, a.vlist, tA + ne, lane);
    __syncwarp();
    // raw candidates: elements >= x0 of the listed vectors (every element of a vector with suppressed ids); the
    // re-reads of up to kRwPre * 32 listed vectors are all in flight before the first is used
    int R = 0;
    for (int e00 = 0; e00 < M; e00 += 32 * kRwPre) {
        uint4 uu[kRwPre];
        int gg[kRwPre];
#pragma unroll
        for (int t = 0; t < kRwPre; ++t) {
            const int e = e00 + 32 * t + lane;
            gg[t] = e < M ? a.vlist[e] : 0;
            uu[t] = e < M ? __ldg(r.row + gg[t]) : neg_inf_vec(VW);
        }
#pragma unroll
        for (int t = 0; t < kRwPre; ++t) {
            if (e00 + 32 * t >= M) break;   // warp-uniform
            const int e = e00 + 32 * t + lane;
            const uint4 u = uu[t];
            const int gv = gg[t];
            uint32_t bits = 0u;
            if (e < M) {
                const bool spec = (gv >= sg.spec_a && gv <= sg.spec_b) || gv == ev;
#pragma unroll
                for (int k = 0; k < VW; ++k)
                    if (spec || vec_elem<VW>(u, k) >= x0) bits |= 1u << k;
            }
            int tot;
            int o = R + warp_excl_i(__popc(bits), lane, tot);
            if (R + tot > kRwRawCap) return false;
#pragma unroll
            for (int k = 0; k < VW; ++k) {
                if ((bits >> k) & 1u) {
                    a.u.raw.v[o] = vec_elem<VW>(u, k);
                    a.u.raw.id[o] = (gv << vsh) + k;
                    ++o;
                }
            }
            R += tot;
        }
    }
    __syncwarp();
    // the history bitmap, built here so that its loads (prefetched into L2 at the row's start) are not waited for
    // ahead of the pass above
    if (r.pen_on && !bm_ready) {
        hist_bad = rw_history(r.hist, r.hlen, r.V, bm, lane);
        bm_ready = true;
    }
    // exact values; the candidates are those >= tau
    int c = 0;
    float m = neg_inf();
    for (int e0 = 0; e0 < R; e0 += 32) {
        const int e = e0 + lane;
        float t = neg_inf();
        int id = 0;
        if (e < R) {
            id = a.u.raw.id[e];
            t = rw_exact(a.u.raw.v[e], id, bm, r);
        }
        const bool keep = e < R && t >= tau;
        const unsigned bal = __ballot_sync(kFull, keep);
        const int pos = c + __popc(bal & ((1u << lane) - 1u));
        if (keep) {
            m = fmaxf(m, t);
            if (pos < kRwCandCap) a.key[pos] = (static_cast<unsigned long long>(okey(t)) << 32) | static_cast<uint32_t>(id);
        }
        c += __popc(bal);
    }
    __syncwarp();
    C = c;
    mx = warp_max_f(m);
    return true;
}

// Step 4: the K-th largest value of the C candidates (a.key, index order; C <= 256, slot s of lane l holds
// position 32 s + l), as an okey, and in `carry_val` an estimate of the value ranked `target` from the top (the next
// row's threshold).  A 64-bucket count linear in [tau, mx] (non-decreasing in the value, so a higher bucket holds
// only larger values) finds the bucket holding the K-th largest; that bucket's members are then ranked exactly.
__device__ uint32_t rw_kth(RwArea& a, int C, int K, int target, float tau, float mx, int lane, float& carry_val) {
    a.bcount[lane] = 0;
    a.bcount[lane + 32] = 0;
    __syncwarp();
    const float span = __fsub_rn(mx, tau);
    const float scale = span > 0.0f ? __fdiv_rn(static_cast<float>(kRankBuckets), span) : 0.0f;
    int bk[kRwSlots];
    uint32_t vk[kRwSlots];
#pragma unroll
    for (int s = 0; s < kRwSlots; ++s) {
        bk[s] = -1;
        vk[s] = 0;
        if (32 * s < C) {
            const int c = 32 * s + lane;
            if (c < C) {
                vk[s] = static_cast<uint32_t>(a.key[c] >> 32);
                bk[s] = min(max(static_cast<int>(__fmul_rn(__fsub_rn(okey_inv(vk[s]), tau), scale)), 0),
                            kRankBuckets - 1);
                atomicAdd(&a.bcount[bk[s]], 1);
            }
        }
    }
    __syncwarp();
    // lane l holds buckets 63 - 2l and 62 - 2l, so the lane prefix runs from the top bucket down
    const int b_hi = kRankBuckets - 1 - 2 * lane, b_lo = b_hi - 1;
    const int n_hi = a.bcount[b_hi], n_lo = a.bcount[b_lo];
    int tot;
    const int above = warp_excl_i(n_hi + n_lo, lane, tot);   // candidates in the buckets above b_hi
    int bstar = -1, need = 0;
    if (above < K && K <= above + n_hi) {
        bstar = b_hi;
        need = K - above;
    } else if (above + n_hi < K && K <= above + n_hi + n_lo) {
        bstar = b_lo;
        need = K - above - n_hi;
    }
    const unsigned w1 = __ballot_sync(kFull, bstar >= 0);   // exactly one lane: 1 <= K <= C
    bstar = __shfl_sync(kFull, bstar, __ffs(w1) - 1);
    need = __shfl_sync(kFull, need, __ffs(w1) - 1);
    // the next threshold: the value ranked `target` from the top, interpolated linearly by rank inside its bucket;
    // with fewer candidates than that, tau moved down by the missing count at the density of the lowest 4 buckets
    int bt = -1, nt = 0, at = 0;
    if (above < target && target <= above + n_hi) {
        bt = b_hi;
        nt = n_hi;
        at = target - above;
    } else if (above + n_hi < target && target <= above + n_hi + n_lo) {
        bt = b_lo;
        nt = n_lo;
        at = target - above - n_hi;
    }
    const unsigned w2 = __ballot_sync(kFull, bt >= 0);
    const int n4 = warp_sum_i(lane >= 30 ? n_hi + n_lo : 0);   // buckets 3..0
    if (scale == 0.0f) {
        carry_val = tau;
    } else if (w2) {
        const int src = __ffs(w2) - 1;
        bt = __shfl_sync(kFull, bt, src);
        nt = __shfl_sync(kFull, nt, src);
        at = __shfl_sync(kFull, at, src);
        // bucket bt spans [tau + bt / scale, tau + (bt + 1) / scale); rank `at` of its nt members, from the top
        const float frac = __fdiv_rn(static_cast<float>(at), static_cast<float>(nt + 1));
        carry_val = __fadd_rn(tau, __fdiv_rn(__fsub_rn(static_cast<float>(bt + 1), frac), scale));
    } else {
        const float per = __fdiv_rn(4.0f, __fmul_rn(static_cast<float>(max(n4, 1)), scale));   // value per candidate
        carry_val = __fsub_rn(tau, __fmul_rn(static_cast<float>(target - C), per));
    }
    // the members of bucket bstar, then the need-th largest of them (ties counted): #(> v) < need <= #(>= v)
    int nb = 0;
#pragma unroll
    for (int s = 0; s < kRwSlots; ++s) {
        if (32 * s < C) {
            const bool in = bk[s] == bstar;
            const unsigned bal = __ballot_sync(kFull, in);
            if (in) a.u.sel.blist[nb + __popc(bal & ((1u << lane) - 1u))] = vk[s];
            nb += __popc(bal);
        }
    }
    __syncwarp();
    uint32_t kth = 0;
    bool found = false;
    for (int j = lane; j < nb; j += 32) {
        const uint32_t v = a.u.sel.blist[j];
        int gt = 0, ge = 0;
        for (int i = 0; i < nb; ++i) {
            const uint32_t w = a.u.sel.blist[i];
            gt += w > v ? 1 : 0;
            ge += w >= v ? 1 : 0;
        }
        if (gt < need && need <= ge) {
            kth = v;
            found = true;
        }
    }
    const unsigned w3 = __ballot_sync(kFull, found);
    return __shfl_sync(kFull, kth, __ffs(w3) - 1);
}

__device__ __forceinline__ unsigned long long warp_sum_ull(unsigned long long v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}

// Step 5: the id, or -1 when a decision lies inside the error band or the survivors do not fit this path (the
// caller replays the row in the reference's order).  Follows Sampler.cs:48-87 on the survivors (the candidates >=
// the K-th largest, ties kept): softmax numerators (libm exp, Sampler.cs:57) in fixed point round(e * 2^52), the
// top-p cut over the ascending (probability, index) order with the last element never removed (:62-72), and the
// inverse-CDF draw over the kept ids in index order (:77-87).  The fixed-point sums are exact; eta = (6 S + 128)
// 2^-53 of the total bounds their difference from the reference's sequential fp64 sums, so a decision farther than
// eta from its threshold is the reference's decision.  Survivor d (index order) sits in slot d >> 5 of lane d & 31.
__device__ int rw_decide(RwArea& a, int C, uint32_t kth, float top_p, double r, float mx, int V, double* out_probs,
                         int lane) {
    // survivors in index order
    int S = 0;
#pragma unroll
    for (int s = 0; s < kRwSlots; ++s) {
        if (32 * s < C) {
            const int c = 32 * s + lane;
            const bool sv = c < C && static_cast<uint32_t>(a.key[c] >> 32) >= kth;
            const unsigned bal = __ballot_sync(kFull, sv);
            const int pos = S + __popc(bal & ((1u << lane) - 1u));
            if (sv && pos < 64) a.u.sel.sv[pos] = a.key[c];
            S += __popc(bal);
        }
    }
    if (S > 64) return -1;
    __syncwarp();
    unsigned long long f[2];
    uint32_t vk[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int d = 32 * h + lane;
        f[h] = 0;
        vk[h] = 0;
        if (d < S) {
            vk[h] = static_cast<uint32_t>(a.u.sel.sv[d] >> 32);
            const double e = softmax_num(okey_inv(vk[h]), mx);   // Sampler.cs:57
            f[h] = __double2ull_rn(__dmul_rn(e, kFix52));
            a.u.sel.e[d] = e;
            a.u.sel.f[d] = f[h];
        }
    }
    const unsigned long long tot = warp_sum_ull(f[0] + f[1]);
    const double eta = (6.0 * S + 128.0) * kU;
    bool kept[2] = {true, true};
    unsigned long long pre_cut = 0;
    if (top_p < 1.0f) {
        // ascending (value, index) order of the survivors = the reference's (probability, index) order, as long
        // as the value groups next to the cut are apart in probability (checked below)
        const uint32_t vmx = okey(mx);
        if (vmx - kth >= (1u << 26)) return -1;   // the 32-bit sort key below would not hold the value
        uint32_t sk[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int d = 32 * h + lane;
            sk[h] = d < S ? (((vk[h] - kth) << 6) | static_cast<uint32_t>(d)) : 0xffffffffu;
        }
        warp_sort32<2>(sk, lane);   // position j = 32 h + lane
#pragma unroll
        for (int h = 0; h < 2; ++h) a.u.sel.sk[32 * h + lane] = sk[h];
        __syncwarp();
        unsigned long long fs[2], inc[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) fs[h] = (32 * h + lane) < S ? a.u.sel.f[sk[h] & 63u] : 0ull;
        inc[0] = warp_incl_ull(fs[0], lane);
        inc[1] = warp_incl_ull(fs[1], lane) + __shfl_sync(kFull, inc[0], 31);
        const double tot_d = static_cast<double>(tot);
        const double thr = static_cast<double>(__fsub_rn(1.0f, top_p));   // Sampler.cs:70, fp32 then widened
        const double T = __dmul_rn(thr, tot_d);
        const double band = __dmul_rn(eta, tot_d);
        int found = -1;
        bool amb = false;
        unsigned long long pc = 0;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int j = 32 * h + lane;
            if (j >= S) continue;
            const double bd = static_cast<double>(inc[h] - fs[h]);   // cum before this element
            const double id = static_cast<double>(inc[h]);           // cum including it
            const bool brk = j <= S - 2 && !(bd > T) && id > T;
            const bool last = j == S - 1 && !(bd > T);
            if (brk || last) {
                found = j;
                pc = inc[h] - fs[h];
                if (brk && !(__dsub_rn(id, T) > band)) amb = true;
                if (bd > 0.0 && !(__dsub_rn(T, bd) > band)) amb = true;
                // the value groups next to the cut must be strictly apart in probability (the reference orders by
                // probability, then index)
                const uint32_t vt = sk[h] >> 6;
                const double et = a.u.sel.e[sk[h] & 63u];
                int jlo = j - 1;
                while (jlo >= 0 && (a.u.sel.sk[jlo] >> 6) == vt) --jlo;
                if (jlo >= 0 && !(a.u.sel.e[a.u.sel.sk[jlo] & 63u] < et * (1.0 - 32.0 * kU))) amb = true;
                if (brk && jlo < j - 1) {   // the cut falls inside this value group: the group above matters too
                    int jhi = j + 1;
                    while (jhi < S && (a.u.sel.sk[jhi] >> 6) == vt) ++jhi;
                    if (jhi < S && !(a.u.sel.e[a.u.sel.sk[jhi] & 63u] > et * (1.0 + 32.0 * kU))) amb = true;
                }
            }
        }
        const unsigned who = __ballot_sync(kFull, found >= 0);
        if (__popc(who) != 1 || __any_sync(kFull, amb)) return -1;
        const int cut = __shfl_sync(kFull, found, __ffs(who) - 1);
        pre_cut = __shfl_sync(kFull, pc, __ffs(who) - 1);
        // kept: the survivors at sorted positions >= cut (Sampler.cs:69 zeroes the ones before)
#pragma unroll
        for (int h = 0; h < 2; ++h)
            if (32 * h + lane < S) a.u.sel.kept[sk[h] & 63u] = (32 * h + lane) >= cut ? 1 : 0;
        __syncwarp();
#pragma unroll
        for (int h = 0; h < 2; ++h) kept[h] = (32 * h + lane) < S && a.u.sel.kept[32 * h + lane] != 0;
    }
    const unsigned long long B = tot - pre_cut;   // mass of the kept survivors (Sampler.cs:73)
    // inverse-CDF draw over the kept ids in index order (Sampler.cs:77-87)
    const double Bd = static_cast<double>(B);
    const double rB = __dmul_rn(r, Bd);
    const double bandB = __dmul_rn(eta, Bd);
    const unsigned long long fk0 = kept[0] ? f[0] : 0ull, fk1 = kept[1] ? f[1] : 0ull;
    const unsigned long long x0 = warp_incl_ull(fk0, lane);
    const unsigned long long x1 = warp_incl_ull(fk1, lane) + __shfl_sync(kFull, x0, 31);
    int hit = -1, hits = 0;
    bool amb = false;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const unsigned long long fc = h == 0 ? fk0 : fk1, hi = h == 0 ? x0 : x1, lo = hi - fc;
        const double lod = static_cast<double>(lo), hid = static_cast<double>(hi);
        if (fc > 0 && !(lod > rB) && hid > rB) {
            ++hits;
            hit = static_cast<int>(static_cast<uint32_t>(a.u.sel.sv[32 * h + lane]));
            if (!(__dsub_rn(hid, rB) > bandB)) amb = true;
            if (lo > 0 && !(__dsub_rn(rB, lod) > bandB)) amb = true;
        }
    }
    hits = warp_sum_i(hits);
    if (hits != 1 || __any_sync(kFull, amb)) return -1;
    const int res = warp_max_i(hit);
    if (out_probs) {
        for (int i = lane; i < V; i += 32) out_probs[i] = 0.0;
        __syncwarp();
        const double scale = __dmul_rn(Bd, 1.0 / kFix52);
#pragma unroll
        for (int h = 0; h < 2; ++h)
            if (kept[h] && 32 * h + lane < S)
                out_probs[static_cast<uint32_t>(a.u.sel.sv[32 * h + lane])] = __ddiv_rn(a.u.sel.e[32 * h + lane], scale);
    }
    return res;
}

// Calls f(raw, id) for every active element of the row: parts A and C (lane l: vectors l, l + 32, ...) and the EOS
// vector (lane 0).  Used by greedy rows and by the threshold rebuild, which need every element's exact value and do
// not depend on the order of the calls.
template <int VW, class F>
__device__ __forceinline__ void rw_for_each(const RwRow& r, const DevSegment& sg, int lane, F f) {
    constexpr int vsh = VW == 4 ? 2 : 3;
#pragma unroll 1
    for (int part = 0; part < 2; ++part) {
        const int v0 = part == 0 ? 0 : sg.c0, nv = part == 0 ? sg.va : sg.vc;
        for (int j0 = 0; j0 < nv; j0 += 32 * kRwBatch) {
            uint4 v[kRwBatch];
#pragma unroll
            for (int i = 0; i < kRwBatch; ++i) {
                const int q = j0 + 32 * i + lane;
                v[i] = q < nv ? __ldg(r.row + v0 + q) : neg_inf_vec(VW);
            }
#pragma unroll
            for (int i = 0; i < kRwBatch; ++i) {
                const int q = j0 + 32 * i + lane;
                if (q < nv) {
#pragma unroll
                    for (int k = 0; k < VW; ++k) f(vec_elem<VW>(v[i], k), ((v0 + q) << vsh) + k);
                }
            }
        }
    }
    if (sg.eosv >= 0 && lane == 0) {
        const uint4 u = __ldg(r.row + sg.eosv);
#pragma unroll
        for (int k = 0; k < VW; ++k) f(vec_elem<VW>(u, k), (sg.eosv << vsh) + k);
    }
}

// A lower threshold for a row that collected 0 < C < K candidates (exact values >= tau, in a.key; C < 64), aimed at
// `target` candidates.  Near tau the counts follow a tail: #(values >= x) ~ C exp((tau - x) / s), with the scale s
// fitted so that the median candidate holds (half of the C above it); tau moves down by s ln(target / C).  (A linear
// step at the density of the smallest candidates overshoots: the density keeps growing below tau.)  Any threshold
// with at least K candidates gives the same decision, so this is only a guess: a row still outside [K, 256] at it goes
// to the whole-row kernel.  Out of line: it runs on misses only.
__device__ __noinline__ float rw_lowered(const RwArea& a, int C, int target, float tau, int lane) {
    uint32_t k[2] = {lane < C ? static_cast<uint32_t>(a.key[lane] >> 32) : 0xffffffffu,
                     lane + 32 < C ? static_cast<uint32_t>(a.key[lane + 32] >> 32) : 0xffffffffu};
    warp_sort32<2>(k, lane);   // ascending values, position p at slot p / 32 of lane p % 32
    const int m = max(1, C >> 1);                                        // m - 1 <= 30: slot 0
    const float gap = okey_inv(__shfl_sync(kFull, k[0], m - 1)) - tau;   // the m-th smallest candidate, above tau
    const float sc = C > m ? gap / logf(static_cast<float>(C) / static_cast<float>(C - m)) : gap;
    return tau - sc * logf(static_cast<float>(target) / static_cast<float>(C));
}

// A threshold tau with at least K exact values >= tau: the K-th largest of the 64 values formed by each lane's two
// largest (a subset of the row, so its K-th largest is <= the row's).  -inf when the row has fewer than K finite
// values among them.
template <int VW>
__device__ __noinline__ float rw_row_threshold(const RwRow& r, const DevSegment& sg, const uint32_t* bm, int K, int lane) {
    float t1 = neg_inf(), t2 = neg_inf();
    rw_for_each<VW>(r, sg, lane, [&](float raw, int id) {
        const float t = rw_exact(raw, id, bm, r);
        t2 = fmaxf(t2, fminf(t1, t));
        t1 = fmaxf(t1, t);
    });
    uint32_t lk[2] = {~okey(t1), ~okey(t2)};   // ascending ~key = descending value
    warp_sort32<2>(lk, lane);
    const uint32_t kk = __shfl_sync(kFull, (K - 1) < 32 ? lk[0] : lk[1], (K - 1) & 31);
    return okey_inv(~kk);
}

// Greedy rows: first index of the maximum of the penalised, masked values (Sampler.cs:90-95); 0 when all are -inf.
template <int VW>
__device__ __noinline__ int rw_argmax(const RwRow& r, const DevSegment& sg, const uint32_t* bm, int lane) {
    float bv = neg_inf();
    int bi = 0x7fffffff;
    rw_for_each<VW>(r, sg, lane, [&](float raw, int id) {
        const float t = rw_exact_greedy(raw, id, bm, r);
        if (t > bv || (t == bv && id < bi)) {
            bv = t;
            bi = id;
        }
    });
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(kFull, bv, off);
        const int oi = __shfl_xor_sync(kFull, bi, off);
        if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
        }
    }
    return is_neg_inf(bv) ? 0 : bi;
}

// One sampling row with 0 < K <= 64 on candidates: the id, or -2 when the row goes to the whole-row kernel.
// `carry` (per lane: segment `lane`'s threshold bits << 32 | option) is read and updated.
template <int VW>
__device__ int rw_sample_row(const LaunchParams& p, const RwRow& r, const DevSegment& sg, const DevOptions& o,
                             RwArea& a, uint32_t* bm, bool& hist_bad, unsigned long long& carry,
                             const unsigned long long* seed, double* out_probs,
                             int lane,
                             uint32_t& st_fast, uint32_t& st_exact, uint32_t& st_miss) {
    const int K = o.top_k;
    const unsigned long long cs = __shfl_sync(kFull, carry, r.seg);
    int C = 0;
    float mx = neg_inf(), tau = neg_inf();
    bool bm_ready = false, have = false;
    if (static_cast<uint32_t>(seed[r.seg]) == static_cast<uint32_t>(r.opt)) {
        // the CTA's seed for this segment and option: the lower eighth of 32 rows' thresholds, which misses far
        // less often than the single row this warp sampled last (that one is the fallback for other options)
        tau = __uint_as_float(static_cast<uint32_t>(seed[r.seg] >> 32));
        have = true;
    } else if (static_cast<uint32_t>(cs) == static_cast<uint32_t>(r.opt)) {
        tau = __uint_as_float(static_cast<uint32_t>(cs >> 32));
        have = true;
    }
    bool ok = false, got = false;
    if (have) {
        const float x0 = raw_threshold(tau, r.inv_t);
        if (fabsf(x0) < pos_inf()) {
            got = rw_collect<VW>(r, sg, tau, x0, bm, bm_ready, hist_bad, a, lane, C, mx);
            ok = got && C >= K && C <= kRwCandCap;
        }
    }
    if (!ok) {   // no usable threshold yet: one more collection, at a threshold that should reach K
        ++st_miss;
        // a few candidates short: the threshold lowered along the tail the candidates show (no pass over the
        // row); otherwise (no threshold, too many candidates) rebuilt from the row's own values.  A lowered
        // threshold that still misses sends the row to the whole-row kernel, so the collection exists twice in the
        // code, not three times.
        const float t2 = got && C > 0 && C < K ? rw_lowered(a, C, K + (K >> 1) + 4, tau, lane) : tau;
        if (t2 < tau) {
            tau = t2;
        } else {
            if (r.pen_on && !bm_ready) {
                hist_bad = rw_history(r.hist, r.hlen, r.V, bm, lane);
                bm_ready = true;
            }
            tau = rw_row_threshold<VW>(r, sg, bm, K, lane);
            if (is_neg_inf(tau)) return -2;   // fewer than K finite values in reach: the whole-row kernel decides
        }
        const float x0 = raw_threshold(tau, r.inv_t);
        if (!(fabsf(x0) < pos_inf())) return -2;
        ok = rw_collect<VW>(r, sg, tau, x0, bm, bm_ready, hist_bad, a, lane, C, mx) && C >= K && C <= kRwCandCap;
        if (!ok) return -2;   // still outside [K, 256] (flat rows, ties): the whole-row kernel decides
    }
    const int target = K + (K >> 1) + 4;
    float gt = tau;
    const uint32_t kth = rw_kth(a, C, K, target, tau, mx, lane, gt);
    int res = p.force_exact ? -1 : rw_decide(a, C, kth, o.top_p, r.uniform, mx, r.V, out_probs, lane);
    if (res >= 0) {
        ++st_fast;
    } else if (C <= kCandCap) {   // a decision inside the error band: the reference's order on the candidates
        res = replay_candidates(a.key, C, K, o, r.uniform, r.V, out_probs, a.u.rflags, lane);
        ++st_exact;
    } else {
        return -2;   // too many candidates for the warp's replay: the whole-row kernel decides the row
    }
    // carry to the next row of this segment: about the value ranked 1.5 K + 4 from the top, so that a similar row
    // collects about that many candidates (rows differ: the window [K, 256] leaves room either way)
    if (!p.force_exact && lane == r.seg && !is_neg_inf(gt) && !isnan(gt))
        carry = (static_cast<unsigned long long>(__float_as_uint(gt)) << 32) | static_cast<uint32_t>(r.opt);
    return res;
}

__device__ __forceinline__ void prefetch_l2(const void* ptr) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(ptr));
}
// Pulls row `row`'s active logit vectors (and its per-row words) into L2, one 128-byte line per lane at a time, so the
// warp's later loads of that row hit L2 instead of waiting on HBM.
__device__ void rw_prefetch_row(const LaunchParams& p, int row, int lane) {
    int s = 0;
    for (int i = 1; i < p.n_segs; ++i)
        if (row >= p.seg[i].row_begin) s = i;
    const DevSegment& sg = p.seg[s];
    if (!sg.rw_ok) return;
    const int local = row - sg.row_begin;
    const unsigned char* base =
        static_cast<const unsigned char*>(sg.logits) + static_cast<int64_t>(local) * sg.row_stride * (sg.dtype == 0 ? 4 : 2);
    for (int b = lane * 128; b < sg.va * 16; b += 32 * 128) prefetch_l2(base + b);
    for (int b = lane * 128; b < sg.vc * 16; b += 32 * 128) prefetch_l2(base + sg.c0 * 16 + b);
    if (lane == 0 && sg.eosv >= 0) prefetch_l2(base + sg.eosv * 16);
    if (lane == 1 && sg.opt_index) prefetch_l2(sg.opt_index + local);
    if (lane == 2 && sg.uniforms) prefetch_l2(sg.uniforms + local);
    if (lane == 3 && sg.kind == 0 && sg.hist_offsets && !sg.hist_lens) prefetch_l2(sg.hist_offsets + local);
    if (lane == 4 && sg.kind == 0 && sg.steps) prefetch_l2(sg.steps + local);
}

// Shared memory of one warp: its RwArea, then its history bitmap ((vmax >> 5) + 1 words, padded to 16 bytes).
__host__ __device__ __forceinline__ int rw_bitmap_words(int vmax) { return (((vmax >> 5) + 1) + 3) & ~3; }
__host__ __device__ __forceinline__ size_t rw_warp_bytes(int vmax) {
    return sizeof(RwArea) + static_cast<size_t>(rw_bitmap_words(vmax)) * 4;
}

// VWK: 4 when every segment of the call holds fp32 rows, 8 when every one holds bf16 rows (the other row path is
// then not compiled into the instance, so the warps fetch half the code), 0 for a mix.
template <int VWK>
__global__ void __launch_bounds__(kRwWarps * 32, 7) row_warp_kernel(const __grid_constant__ LaunchParams p) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int lane = threadIdx.x & 31;
    const int wib = threadIdx.x >> 5;
    unsigned char* mine = smem + static_cast<size_t>(wib) * rw_warp_bytes(p.vmax);
    RwArea& a = *reinterpret_cast<RwArea*>(mine);
    uint32_t* bm = reinterpret_cast<uint32_t*>(mine + sizeof(RwArea));
    // launched as a programmatic dependent of the stream's previous kernel: its results are visible from here on
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // the whole-row kernel may be scheduled now; it waits (griddepcontrol.wait) until this grid has finished
    if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // the first row's logits and per-row words start towards L2 before the seed table is read
    if (blockIdx.x * kRwWarps + wib < p.total_rows) rw_prefetch_row(p, blockIdx.x * kRwWarps + wib, lane);

    const int G = gridDim.x * kRwWarps;
    // carried thresholds: lane s holds segment s's (threshold bits << 32 | option); ~0: none yet
    unsigned long long carry = ~0ull;
    // the CTA's seeds, one per segment: the lower eighth (the 4th lowest of 32: robust to an atypical row, and low
    // enough that rows a little below the typical one still reach K) of the thresholds the last call's warps left in
    // the table for that segment, among those of the option the segment's first slot holds
    __shared__ unsigned long long seed[kMaxSegments];
    if (wib < p.n_segs) {
        unsigned long long e = p.guess_seed ? p.guess_seed[wib * kSeedSlots + lane] : ~0ull;
        const uint32_t opt0 = __shfl_sync(kFull, static_cast<uint32_t>(e), 0);
        const bool m = static_cast<uint32_t>(e) == opt0 && opt0 != 0xffffffffu &&
                       !isnan(__uint_as_float(static_cast<uint32_t>(e >> 32)));
        uint32_t kk[1] = {m ? okey(__uint_as_float(static_cast<uint32_t>(e >> 32))) : 0xffffffffu};
        const int n = __popc(__ballot_sync(kFull, m));
        warp_sort32<1>(kk, lane);
        const uint32_t q = __shfl_sync(kFull, kk[0], max(n - 1, 0) >> 3);
        if (lane == 0) seed[wib] = n > 0 ? ((static_cast<unsigned long long>(__float_as_uint(okey_inv(q))) << 32) | opt0) : ~0ull;
    }
    for (int s2 = kRwWarps + wib; s2 < p.n_segs; s2 += kRwWarps)   // more segments than warps: no seed
        if (lane == 0) seed[s2] = ~0ull;
    __syncthreads();
    uint32_t st_greedy = 0, st_fast = 0, st_exact = 0, st_overflow = 0, st_miss = 0;

    for (int row = blockIdx.x * kRwWarps + wib; row < p.total_rows; row += G) {
        int s = 0;
        for (int i = 1; i < p.n_segs; ++i)
            if (row >= p.seg[i].row_begin) s = i;
        const DevSegment& sg = p.seg[s];
        const int local = row - sg.row_begin;
        // the row's own words, one lane each
        long long w = 0;
        if (lane == 0) w = sg.opt_index ? sg.opt_index[local] : 0;
        if (lane == 1) w = (sg.kind == 0 && sg.steps) ? sg.steps[local] : 0x7fffffff;
        if (lane == 2) w = sg.uniforms ? __double_as_longlong(sg.uniforms[local]) : 0;
        if (lane == 3 || lane == 4) {
            int64_t b0 = 0, b1 = 0;
            row_history(sg, local, b0, b1);
            w = lane == 3 ? b0 : b1;
        }
        if (lane == 5) w = sg.active ? sg.active[local] : 1;
        if (__shfl_sync(kFull, w, 5) == 0) {   // a device-resident batch's finished slot: no sample
            if (lane == 0) sg.out_ids[local] = -1;
            continue;
        }
        const int opt = static_cast<int>(__shfl_sync(kFull, w, 0));
        const int step = static_cast<int>(__shfl_sync(kFull, w, 1));
        const double uniform = __longlong_as_double(__shfl_sync(kFull, w, 2));
        long long hb = __shfl_sync(kFull, w, 3), he = __shfl_sync(kFull, w, 4);
        if (hb < 0 || he < hb) {   // device-memory offsets are checked here: report, and read no history
            if (lane == 0) atomicOr(p.err, kErrHistOffsets);
            hb = he = 0;
        }
        int32_t* out_id = sg.out_ids + local;
        if (opt < 0 || opt >= p.n_opts) {
            if (lane == 0) {
                atomicOr(p.err, kErrBadOption);
                *out_id = -1;
            }
            continue;
        }
        const DevOptions o = p.n_opts <= kInlineOptions ? p.inl_opts[opt] : p.dev_opts[opt];
        const int V = sg.vocab;
        const bool pen_on = sg.kind == 0 && o.rep_penalty != 1.0f && he > hb;
        const bool sample = o.do_sample != 0;
        const bool defer = !sg.rw_ok || (sample && !(o.top_k > 0 && o.top_k < V && o.top_k <= kSmallK)) ||
                           (pen_on && !(o.rep_penalty >= 1.0f));
        if (defer) {
            if (lane == 0) p.deferred_rows[atomicAdd(p.deferred_count, 1u)] = row;
            continue;
        }
        RwRow r;
        r.row = reinterpret_cast<const uint4*>(static_cast<const unsigned char*>(sg.logits) +
                                              static_cast<int64_t>(local) * sg.row_stride * (sg.dtype == 0 ? 4 : 2));
        r.uniform = uniform;
        r.pen = o.rep_penalty;
        const bool inl = p.n_opts <= kInlineOptions;
        r.pen_rcp = !pen_on ? 1.0 : inl ? p.inl_pen_rcp[opt] : __drcp_rn(static_cast<double>(o.rep_penalty));
        r.inv_t = !sample ? 1.0f : inl ? p.inl_inv_t[opt] : __fdiv_rn(1.0f, o.temperature);
        r.row_id = row;
        r.seg = s;
        r.opt = opt;
        r.local = local;
        r.V = V;
        r.kind = sg.kind;
        r.sup_lo = sg.sup_lo;
        r.sup_hi = sg.sup_hi;
        r.eos = sg.eos;
        r.eos_blocked = sg.kind == 0 && step < sg.min_new;
        r.pen_on = pen_on;
        double* out_probs = sg.out_probs ? sg.out_probs + static_cast<int64_t>(local) * V : nullptr;
        r.hist = sg.hist_ids + hb;
        r.hlen = static_cast<int>(he - hb);
        if (pen_on)   // into L2 now; read when the bitmap is built
            for (int j = lane * 32; j < r.hlen; j += 32 * 32) prefetch_l2(r.hist + j);
        if (row + G < p.total_rows) rw_prefetch_row(p, row + G, lane);   // this warp's next row

        bool hist_bad = false;
        int res;
        if (!sample) {
            if (pen_on) hist_bad = rw_history(r.hist, r.hlen, V, bm, lane);
            res = (VWK == 4 || (VWK == 0 && sg.dtype == 0)) ? rw_argmax<4>(r, sg, bm, lane) : rw_argmax<8>(r, sg, bm, lane);
            if (out_probs)
                for (int i = lane; i < V; i += 32) out_probs[i] = 0.0;
            ++st_greedy;
        } else {
            res = (VWK == 4 || (VWK == 0 && sg.dtype == 0))
                      ? rw_sample_row<4>(p, r, sg, o, a, bm, hist_bad, carry, seed, out_probs, lane, st_fast,
                                                   st_exact, st_miss)
                                : rw_sample_row<8>(p, r, sg, o, a, bm, hist_bad, carry, seed, out_probs, lane, st_fast,
                                                   st_exact, st_miss);
        }
        // seeds the next call: slot j of segment s holds the threshold carried out of row j of s (one writer per
        // slot, so the table is the same whatever order the warps finish in)
        if (sample && p.guess_seed && local < kSeedSlots && lane == s && carry != ~0ull)
            p.guess_seed[lane * kSeedSlots + local] = carry;
        if (hist_bad && lane == 0) atomicOr(p.err, kErrHistRange);
        if (res == -2) {   // the whole-row kernel takes the row
            ++st_overflow;
            if (lane == 0) p.deferred_rows[atomicAdd(p.deferred_count, 1u)] = row;
        } else if (lane == 0) {
            *out_id = res;
        }
        __syncwarp();   // the warp's shared area is reused by its next row
    }
    if (p.stats && lane == 0) {
        const uint32_t v[4] = {st_greedy, st_fast, st_exact, st_overflow};
        const int idx[4] = {kStatGreedy, kStatFast, kStatFastReplayed, kStatOverflow};
        for (int i = 0; i < 4; ++i)
            if (v[i]) atomicAdd(&p.stats[idx[i]], static_cast<unsigned long long>(v[i]));
        if (st_miss) atomicAdd(&p.stats[kStatThresholdMiss], static_cast<unsigned long long>(st_miss));
    }
}
