// qsamp_hist.cuh -- the histogram path for bf16 full-vocabulary rows
// (included by qsamp_kernels.cu inside namespace qs).
//
// A bf16 row holds at most 65536 distinct values, and after the row
// transform (soft-cap, /T; both monotone) every element outside the penalty
// window has the value of its bf16 pattern. The row sorted as the reference
// sorts it (sampling.cpp:158-163: value descending; equal values here by
// ascending id) is therefore a sequence of GROUPS of equal values, and each
// of the reference's sequential float sums (sum_exp :171, the cumulative
// top-p sum :173-178, the softmax sum :184-188, and the double partial sums
// of std::discrete_distribution :192-193) adds runs of equal terms, which
// qs_run_add / qs_run_add_d add exactly in O(1) per binade. The row is read
// from HBM once, into a histogram of its 65536 bf16 keys in shared memory;
// no element is sorted.
//
// One CTA (512 threads) per row, rows from a queue:
//   1. the penalty window's distinct ids (a hash table with counts);
//   2. one pass over the row: allow-mask, histogram by the order-preserving
//      16-bit key (two 16-bit counts per shared-memory word);
//   3. the total count exposes an overflowed bin; the window's elements get
//      their penalised values and leave the histogram;
//   4. the row max M (the largest key still counted, and the window);
//   5. groups: the keys with elements and a value within 17.5 of M (below,
//      expf(x - M) < 2^-25, which no sum sees), merged with the window's
//      elements, in descending value;
//   6. the three sums as scans over groups: each group's run is added by
//      qs_run_add from a guess of the running sum at its start, the prefix of
//      the exact increments gives the next guesses, and the scan repeats
//      until no start changes (each pass fixes at least the first wrong start;
//      two or three passes in practice);
//   7. the drawn position's group, its rank among the row's elements of that
//      value, and the element of that rank (ascending id): a scan of the row.
// A row this path does not prove exact -- a NaN or infinite pattern, a bin
// past 65535, more than HS_GMAX groups, a scan that does not settle, a cut
// below the groups, probabilities too small for an exact double normaliser
// -- goes to a device-side list that the cluster kernel serves next; no row
// is answered approximately.

constexpr int HS_NT = NT;            // threads per CTA (the block helpers' width)
constexpr int HS_GMAX = 4096;        // groups walked per row
constexpr int HS_GPT = HS_GMAX / HS_NT;
constexpr int HS_DMAX = 2048;        // survivor groups of the draw
constexpr int HS_WMAX = 1024;        // penalty window served
constexpr int HS_HT = 2048;          // window hash slots
constexpr int HS_ITERS = 24;         // scan passes before a row is handed on
constexpr float HS_DMIN = -17.5f;    // x - M below this: expf < 2^-25, no sum sees it
constexpr int HS_LD = 8;             // 16-byte loads in flight per thread in the histogram pass
constexpr int HS_KLO = 128, HS_KHI = 65408;  // keys of finite bf16 values: [HS_KLO, HS_KHI)
static_assert(HS_GMAX % HS_NT == 0 && HS_DMAX % HS_NT == 0, "groups per thread");

struct HsLayout {
    int off_hist, off_gx, off_gc, off_gt, off_hid, off_hcnt, off_wx, off_wid, off_exp, off_misc, total;
};
__host__ __device__ inline HsLayout hs_layout() {
    HsLayout L;
    int o = 0;
    L.off_hist = o; o = align_up(o + 65536 * 2, 16);          // u16 counts by key; the walks' arrays after step 5
    L.off_gx = o;   o = align_up(o + HS_GMAX * 4, 16);        // group value x
    L.off_gc = o;   o = align_up(o + HS_GMAX * 4, 16);        // group count
    L.off_gt = o;   o = align_up(o + HS_GMAX * 4, 16);        // group term (t, then q, then p)
    L.off_hid = o;  o = align_up(o + HS_HT * 4, 16);          // window hash: ids
    L.off_hcnt = o; o = align_up(o + HS_HT * 4, 16);          //   counts
    L.off_wx = o;   o = align_up(o + HS_WMAX * 4, 16);        // distinct window ids' values
    L.off_wid = o;  o = align_up(o + HS_WMAX * 4, 16);        //   and ids
    L.off_exp = o;  o = align_up(o + 32 * 8, 16);
    L.off_misc = o; o = align_up(o + (int)sizeof(Misc), 16);
    L.total = o;
    return L;
}
// The walks' arrays inside the histogram's 128 KB (byte offsets), free once
// the groups are built:
//   walks A/B: sA float[GMAX] 0 | inc u64[GMAX] 16K | sB float[GMAX] 48K | stp int[GMAX] 64K
//   all along: pref u64[GMAX] 80K (group start positions) | wk u64[WMAX] 112K (window keys)
//   until the sums: the window keys in descending order, u64[WMAX] 16K
//   the draw (after sum_keep): inc2 u128[DMAX] 0 | wd double[DMAX] 32K | sC double[DMAX] 48K
//              | stp (first DMAX) 64K | gcd u32[DMAX] 120K
//   the recovery: wm int[WMAX] 0
enum : int {
    HO_SA = 0, HO_INC = 16384, HO_SB = 49152, HO_STP = 65536, HO_PREF = 81920, HO_WK = 114688,
    HO_INC2 = 0, HO_WD = 32768, HO_SC = 49152, HO_GCD = 122880, HO_WM = 0,
};
static_assert(HO_WK + HS_WMAX * 8 <= HO_GCD && HO_GCD + HS_DMAX * 4 <= 131072, "walk arrays overlap");

// The order-preserving 16-bit key of a bf16 pattern and back.
__device__ __forceinline__ uint32_t hs_key(uint32_t p) { return (p & 0x8000u) ? (~p & 0xffffu) : (p | 0x8000u); }
__device__ __forceinline__ uint32_t hs_pat(uint32_t k) { return (k & 0x8000u) ? (k & 0x7fffu) : (~k & 0xffffu); }

// The transformed value of a non-window, allowed element with key k
// (soft-cap, /T, canon: monotone non-decreasing over finite keys).
__device__ __forceinline__ float hs_value(const RowCtx& r, uint32_t k) {
    const uint32_t p = hs_pat(k);
    float v = qs_bf16_to_f32((uint16_t)p);
    if (r.cap_on) v = r.lut ? r.lut[p] : qs_softcap(v, r.cap);
    return post_value(r, v);
}
__device__ __forceinline__ uint32_t hs_count(const uint32_t* hist, int k) {
    return (hist[k >> 1] >> ((k & 1) << 4)) & 0xffffu;
}

struct HsMisc {
    float M, S1, S2;
    int nuniq, bail, changed, top_key, found_id, nwm, next_ri, kmin, klo, khi;
};

// The smallest k in [lo, hi) with pred(k), or hi, for a pred that is false
// and then true over the range: a 32-way search by one warp (every lane gets
// the answer). The smallest such k stays in [lo, hi] (hi: none); each round
// tests 31 points evenly spread over the range, the last standing for hi.
template <typename P>
__device__ int hs_warp_search(int lo, int hi, P pred) {
    const int lane = threadIdx.x & 31;
    while (hi - lo > 32) {
        const int pt = lo + (int)(((long long)(hi - lo) * (lane + 1)) / 32);  // lane 31: hi
        const bool t = pt < hi && pred(pt);
        const uint32_t bt = __ballot_sync(FULLMASK, t) | 0x80000000u;
        const int f = __ffs(bt) - 1;  // first point at which pred holds (31: hi)
        const int pf = lo + (int)(((long long)(hi - lo) * (f + 1)) / 32);
        const int pp = f > 0 ? lo + (int)(((long long)(hi - lo) * f) / 32) + 1 : lo;
        lo = pp;
        hi = pf;
    }
    const int kk = lo + lane;
    const uint32_t bt = __ballot_sync(FULLMASK, kk < hi && pred(kk));
    return bt ? lo + __ffs(bt) - 1 : hi;
}

// Exclusive scan, in place, of n <= HS_GMAX u64 values; returns the total.
// Thread t owns entries [t*HS_GPT, (t+1)*HS_GPT).
__device__ unsigned long long hs_scan_u64(unsigned long long* a, int n, unsigned long long* wtot) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    unsigned long long v[HS_GPT], s = 0;
#pragma unroll
    for (int e = 0; e < HS_GPT; ++e) {
        const int j = threadIdx.x * HS_GPT + e;
        v[e] = j < n ? a[j] : 0ull;
        s += v[e];
    }
    unsigned long long x = s;
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long y = __shfl_up_sync(FULLMASK, x, o);
        if (lane >= o) x += y;
    }
    __syncthreads();
    if (lane == 31) wtot[w] = x;
    __syncthreads();
    if (w == 0) {
        unsigned long long q = lane < NWARPS ? wtot[lane] : 0ull;
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned long long y = __shfl_up_sync(FULLMASK, q, o);
            if (lane >= o) q += y;
        }
        if (lane < NWARPS) wtot[lane] = q;
    }
    __syncthreads();
    unsigned long long run = (w > 0 ? wtot[w - 1] : 0ull) + x - s;
    const unsigned long long total = wtot[NWARPS - 1];
#pragma unroll
    for (int e = 0; e < HS_GPT; ++e) {
        const int j = threadIdx.x * HS_GPT + e;
        if (j < n) a[j] = run;
        run += v[e];
    }
    __syncthreads();
    return total;
}

// The same for unsigned 128-bit values over n <= HS_DMAX entries (the
// draw's cumulative weights).
typedef unsigned __int128 u128;
constexpr int HS_DPT = HS_DMAX / HS_NT;
__device__ __forceinline__ u128 shfl_up_u128(u128 x, int o) {
    const unsigned long long lo = __shfl_up_sync(FULLMASK, (unsigned long long)x, o);
    const unsigned long long hi = __shfl_up_sync(FULLMASK, (unsigned long long)(x >> 64), o);
    return ((u128)hi << 64) | lo;
}
__device__ void hs_scan_u128(u128* a, int n, u128* wtot) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    u128 v[HS_DPT], s = 0;
#pragma unroll
    for (int e = 0; e < HS_DPT; ++e) {
        const int j = threadIdx.x * HS_DPT + e;
        v[e] = j < n ? a[j] : (u128)0;
        s += v[e];
    }
    u128 x = s;
    for (int o = 1; o < 32; o <<= 1) {
        const u128 y = shfl_up_u128(x, o);
        if (lane >= o) x += y;
    }
    __syncthreads();
    if (lane == 31) wtot[w] = x;
    __syncthreads();
    if (w == 0) {
        u128 q = lane < NWARPS ? wtot[lane] : (u128)0;
        for (int o = 1; o < 32; o <<= 1) {
            const u128 y = shfl_up_u128(q, o);
            if (lane >= o) q += y;
        }
        if (lane < NWARPS) wtot[lane] = q;
    }
    __syncthreads();
    u128 run = (w > 0 ? wtot[w - 1] : (u128)0) + x - s;
#pragma unroll
    for (int e = 0; e < HS_DPT; ++e) {
        const int j = threadIdx.x * HS_DPT + e;
        if (j < n) a[j] = run;
        run += v[e];
    }
    __syncthreads();
}

// A float as a count of 2^-sh units (f >= 0; exact when f is a multiple of
// 2^-sh, else truncated) and back (the nearest float).
__device__ __forceinline__ unsigned long long f_units(float f, int sh) {
    const uint32_t b = __float_as_uint(f);
    const int e = (int)(b >> 23);
    if (e == 0) return 0ull;  // zero (the walks hold no subnormal sums)
    const unsigned long long mnt = (unsigned long long)((b & 0x7fffffu) | 0x800000u);
    const int s = e - 150 + sh;  // f = mnt * 2^(e - 150)
    return s >= 0 ? (mnt << s) : (s > -64 ? (mnt >> (-s)) : 0ull);
}
__device__ __forceinline__ float units_f(unsigned long long u, int sh) {
    return __fmul_rn(__ull2float_rn(u), __uint_as_float((uint32_t)(127 - sh) << 23));
}
// A double as a count of 2^-96 units (0 <= d < 2^31) and back.
__device__ __forceinline__ u128 d_units(double d) {
    const unsigned long long b = (unsigned long long)__double_as_longlong(d);
    const int e = (int)(b >> 52);
    if (e == 0) return 0;
    const u128 mnt = (u128)((b & ((1ull << 52) - 1ull)) | (1ull << 52));
    const int s = e - 1075 + 96;
    return s >= 0 ? (mnt << s) : (s > -128 ? (mnt >> (-s)) : (u128)0);
}
__device__ __forceinline__ double units_d(u128 u) {
    // the nearest double to u * 2^-96 (exact for a double's units: each half
    // holds at most 53 significant bits, and the fma rounds once)
    const unsigned long long hi = (unsigned long long)(u >> 64), lo = (unsigned long long)u;
    return __fma_rn(__ull2double_rn(hi), 0x1p-32, __dmul_rn(__ull2double_rn(lo), 0x1p-96));
}

// One sequential float sum over groups g < n as a scan: term[g] added cnt[g]
// times from start[g] (guessed on entry), until no start changes. Units of
// 2^-sh hold every running sum exactly. The first add reaching `stop` ends
// the sum; stop_at[g] receives the index of that add inside group g (or
// cnt[g]). Returns false when the scan did not settle in HS_ITERS passes.
__device__ bool hs_walk_f(int n, const uint32_t* cnt, const float* term, float* start, unsigned long long* incr,
                          int* stop_at, float stop, int sh, unsigned long long* wtot, HsMisc* hm, int* iters = nullptr) {
    for (int it = 0; it < HS_ITERS; ++it) {
        if (iters) *iters = it + 1;
        for (int g = threadIdx.x; g < n; g += HS_NT) {
            float S = start[g];
            const long long at = qs_run_add(&S, term[g], (long long)cnt[g], stop);
            if (stop_at) stop_at[g] = (int)at;
            incr[g] = f_units(S, sh) - f_units(start[g], sh);
        }
        if (threadIdx.x == 0) hm->changed = 0;
        __syncthreads();
        const unsigned long long base = f_units(start[0], sh);
        hs_scan_u64(incr, n, wtot);
        int ch = 0;
        for (int g = threadIdx.x; g < n; g += HS_NT) {
            const float s2 = units_f(base + incr[g], sh);
            if (s2 != start[g]) ch = 1;
            start[g] = s2;
        }
        if (ch) hm->changed = 1;
        __syncthreads();
        const bool done = !hm->changed;
        __syncthreads();
        if (done) return true;
    }
    return false;
}

// The same in double (units of 2^-96, 128-bit prefix sums), n <= HS_DMAX.
__device__ bool hs_walk_d(int n, const uint32_t* cnt, const double* term, double* start, u128* incr, int* stop_at,
                          double stop, u128* wtot, HsMisc* hm, int* iters = nullptr) {
    for (int it = 0; it < HS_ITERS; ++it) {
        if (iters) *iters = it + 1;
        for (int g = threadIdx.x; g < n; g += HS_NT) {
            double S = start[g];
            const long long at = qs_run_add_d(&S, term[g], (long long)cnt[g], stop);
            stop_at[g] = (int)at;
            incr[g] = d_units(S) - d_units(start[g]);
        }
        if (threadIdx.x == 0) hm->changed = 0;
        __syncthreads();
        const u128 base = d_units(start[0]);
        hs_scan_u128(incr, n, wtot);
        int ch = 0;
        for (int g = threadIdx.x; g < n; g += HS_NT) {
            const double s2 = units_d(base + incr[g]);
            if (s2 != start[g]) ch = 1;
            start[g] = s2;
        }
        if (ch) hm->changed = 1;
        __syncthreads();
        const bool done = !hm->changed;
        __syncthreads();
        if (done) return true;
    }
    return false;
}

// The penalty window of a row (sampling.cpp:124-129 with the frequency /
// presence extension): its distinct ids in wid[0, hm.nuniq), each with its
// count in an open-addressing table (hid / hcnt, HS_HT slots, cleared here).
// A window longer than HS_WMAX sets hm.bail. Ends with a barrier.
__device__ void hs_window(const QsLaunch& a, int row, const qsamp_row_params& p, int V, int32_t* hid, int32_t* hcnt,
                          int32_t* wid, HsMisc& hm) {
    for (int q = threadIdx.x; q < HS_HT; q += HS_NT) {
        hid[q] = -1;
        hcnt[q] = 0;
    }
    __syncthreads();
    const bool rep_on = p.repetition_penalty != 1.0f;
    const bool fp_on = p.frequency_penalty != 0.0f || p.presence_penalty != 0.0f;
    if ((rep_on || fp_on) && a.hist) {
        const int len = a.hist_len ? a.hist_len[row] : a.hist_stride;
        const unsigned long long lb = (unsigned long long)(long long)p.repetition_lookback;
        const int wl = len > 0 ? (int)(lb < (unsigned long long)len ? lb : (unsigned long long)len) : 0;
        if (wl > HS_WMAX) {
            if (threadIdx.x == 0) hm.bail = 1;
        } else {
            const int32_t* h = a.hist + (size_t)row * (size_t)a.hist_stride + (len - wl);
            for (int j = threadIdx.x; j < wl; j += HS_NT) {
                const int32_t id = h[j];
                if (id < 0 || id >= V) continue;
                uint32_t slot = ((uint32_t)id * 2654435761u) & (HS_HT - 1);
                while (true) {  // at most HS_WMAX <= HS_HT / 2 distinct ids: a free slot exists
                    const int old = atomicCAS(&hid[slot], -1, id);
                    if (old == -1 || old == id) {
                        if (atomicAdd(&hcnt[slot], 1) == 0) wid[atomicAdd(&hm.nuniq, 1)] = id;
                        break;
                    }
                    slot = (slot + 1) & (HS_HT - 1);
                }
            }
        }
    }
    __syncthreads();
}
// The count of window id `id` (present in the table).
__device__ __forceinline__ int hs_window_count(const int32_t* hid, const int32_t* hcnt, int id) {
    uint32_t slot = ((uint32_t)id * 2654435761u) & (HS_HT - 1);
    while (hid[slot] != id) slot = (slot + 1) & (HS_HT - 1);
    return hcnt[slot];
}
// The penalised value of window element v (after the soft-cap and the
// allow-mask: -inf when masked), then /T and canon (sampling.cpp:130-135,
// 154-156).
__device__ __forceinline__ float hs_penalise(const RowCtx& r, const qsamp_row_params& p, float v, int c) {
    if (p.repetition_penalty != 1.0f)
        v = v < 0.0f ? __fmul_rn(v, p.repetition_penalty) : __fdiv_rn(v, p.repetition_penalty);
    if (p.frequency_penalty != 0.0f || p.presence_penalty != 0.0f) {
        v = __fsub_rn(v, __fmul_rn((float)c, p.frequency_penalty));
        v = __fsub_rn(v, p.presence_penalty);
    }
    return post_value(r, v);
}

// The scratch arrays of the sums and the draw (inside the histogram's 128 KB
// in both kernels that use them).
struct HsArrays {
    float* sA;
    unsigned long long* inc;
    float* sB;
    int* stp;
    unsigned long long* pref;  // group start positions (set by the caller)
    u128* inc2;
    double* wd;
    double* sC;
    uint32_t* gcd;
};
__device__ __forceinline__ HsArrays hs_arrays(unsigned char* H) {
    HsArrays w;
    w.sA = (float*)(H + HO_SA);
    w.inc = (unsigned long long*)(H + HO_INC);
    w.sB = (float*)(H + HO_SB);
    w.stp = (int*)(H + HO_STP);
    w.pref = (unsigned long long*)(H + HO_PREF);
    w.inc2 = (u128*)(H + HO_INC2);
    w.wd = (double*)(H + HO_WD);
    w.sC = (double*)(H + HO_SC);
    w.gcd = (uint32_t*)(H + HO_GCD);
    return w;
}
// What the sums and the draw give: the row's sums, the kept count, the drawn
// sorted position, its group and probability.
struct HsDrawn {
    float S1, S2, prob;
    long long n_keep, pos;
    int gp, jc, it_s, it_c, it_d;
};

// The reference's sums and draw over the row's groups (gx: values in
// descending order, gc: counts, w.pref: start positions, G <= HS_GMAX groups
// that hold every element within HS_DMIN of the maximum M). gt is scratch.
// Returns false when the row cannot be proven exact here (a scan that does
// not settle, a cut below the groups, too many survivor groups, a normaliser
// that is not exact in double); the caller hands it on.
__device__ bool hs_sums_draw(const QsLaunch& a, int row, const qsamp_row_params& p, int G, const float* gx,
                             const uint32_t* gc, float* gt, const HsArrays& w, const uint64_t* exp32, float M,
                             HsMisc& hm, unsigned long long* wtot, u128* wtot2, Misc* m, HsDrawn& o) {
    const float POS_INF = __int_as_float(0x7f800000);
    float* const sA = w.sA;
    unsigned long long* const inc = w.inc;
    float* const sB = w.sB;
    int* const stp = w.stp;
    const unsigned long long* const pref = w.pref;
    // ---- sum_exp: t = expf(x - M) in sorted order (sampling.cpp:171)
    for (int g = threadIdx.x; g < G; g += HS_NT) gt[g] = qs_expf_tab(__fsub_rn(gx[g], M), exp32);
    __syncthreads();
    // starts guessed from the exact masses (a prefix of count * t)
    for (int g = threadIdx.x; g < G; g += HS_NT) inc[g] = (unsigned long long)gc[g] * f_units(gt[g], 30);
    __syncthreads();
    hs_scan_u64(inc, G, wtot);
    for (int g = threadIdx.x; g < G; g += HS_NT) sA[g] = g == 0 ? 0.0f : units_f(inc[g], 30);
    __syncthreads();
    QS_TMARK(row, 19, true);
    o.it_s = o.it_c = o.it_d = 0;
    // Groups whose term is below half an ulp of the running sum add nothing,
    // and neither does any later one (smaller terms, a larger sum): the walk
    // covers the groups before the first whose term is below a quarter ulp
    // of its guessed start (the float sum stays within a factor 2 of the
    // real-valued one), checks the bound at the exact sum it reaches, and
    // walks every group if the check fails.
    int nlive = G;
    for (int g = threadIdx.x; g < G; g += HS_NT) {
        const uint32_t sb = __float_as_uint(sA[g]);
        if (g > 0 && sb >= (26u << 23) && gt[g] < __uint_as_float((sb & 0x7f800000u) - (25u << 23))) nlive = min(nlive, g);
    }
    nlive = block_min_int(nlive, m);
    while (true) {
        if (!hs_walk_f(nlive, gc, gt, sA, inc, nullptr, POS_INF, 23, wtot, &hm, &o.it_s)) return false;
        if (threadIdx.x == 0) {
            float S = sA[nlive - 1];
            qs_run_add(&S, gt[nlive - 1], (long long)gc[nlive - 1], POS_INF);
            hm.S1 = S;
            // the first group left out must be below half an ulp of the sum
            const uint32_t sb = __float_as_uint(S);
            hm.changed = nlive < G && !(gt[nlive] < __uint_as_float((sb & 0x7f800000u) - (24u << 23)));
        }
        __syncthreads();
        if (!hm.changed || nlive == G) break;
        nlive = G;  // (the starts walked so far are exact; the rest keep their guesses)
        __syncthreads();
    }
    const float S1 = hm.S1;
    // the starts of the groups left out: the final sum (sum_keep reads them)
    for (int g = nlive + threadIdx.x; g < G; g += HS_NT) sA[g] = S1;
    __syncthreads();
    QS_TMARK(row, 5, true);

    // ---- the top-p cut: cum += t / sum_exp until cum >= top_p (:173-178)
    for (int g = threadIdx.x; g < G; g += HS_NT) {
        gt[g] = __fdiv_rn(gt[g], S1);
        inc[g] = (unsigned long long)gc[g] * f_units(gt[g], 52);
    }
    __syncthreads();
    hs_scan_u64(inc, G, wtot);
    for (int g = threadIdx.x; g < G; g += HS_NT) sB[g] = g == 0 ? 0.0f : units_f(inc[g], 52);
    __syncthreads();
    // The cut lies before the first group whose exact (real-valued) start
    // reaches top_p + 1/64 -- the float sum drifts from the exact one by far
    // less -- and no later group changes the sums before it: the walk covers
    // those groups, and all of them only if it finds no cut there.
    int nwalk = G;
    {
        const float thr = __fadd_rn(p.top_p, 0.015625f);
        for (int g = threadIdx.x; g < G; g += HS_NT)
            if (sB[g] >= thr) nwalk = min(nwalk, g);
        nwalk = max(1, block_min_int(nwalk, m));
    }
    int jc = G;  // the cut group: the first whose sum stopped inside it
    while (true) {
        if (!hs_walk_f(nwalk, gc, gt, sB, inc, stp, p.top_p, 60, wtot, &hm, &o.it_c)) return false;
        jc = G;
        for (int g = threadIdx.x; g < nwalk; g += HS_NT)
            if ((uint32_t)stp[g] < gc[g]) jc = min(jc, g);
        jc = block_min_int(jc, m);
        if (jc < G || nwalk == G) break;
        nwalk = G;  // (the starts walked so far are exact; the rest keep their guesses)
    }
    if (jc >= G || jc >= HS_DMAX) return false;  // a cut below the groups, or too many survivor groups
    const int sc = stp[jc];  // index of the cutting add inside group jc
    const long long n_keep = (long long)pref[jc] + sc + 1;
    // sum_keep: the first n_keep terms of the sum_exp order (:184-188)
    for (int g = threadIdx.x; g <= jc; g += HS_NT) gt[g] = qs_expf_tab(__fsub_rn(gx[g], M), exp32);
    __syncthreads();
    if (threadIdx.x == 0) {
        float S = sA[jc];
        qs_run_add(&S, gt[jc], (long long)sc + 1, POS_INF);
        hm.S2 = S;
    }
    __syncthreads();
    const float S2 = hm.S2;
    QS_TMARK(row, 6, true);
    // probabilities p = t / sum_keep (:189) over the survivor groups
    const int ng = jc + 1;
    for (int g = threadIdx.x; g < ng; g += HS_NT) gt[g] = __fdiv_rn(gt[g], S2);
    __syncthreads();

    // ---- the draw (std::discrete_distribution, :192-193)
    long long pos = 0;
    if (n_keep >= 2) {
        // the normaliser, the probabilities summed in double: exact (every
        // partial sum a multiple of 2^-52 below 2) when the smallest
        // probability is at least 2^-29
        if (!(gt[jc] >= 0x1p-29f)) return false;
        u128* const inc2 = w.inc2;
        double* const wd = w.wd;
        double* const sC = w.sC;
        uint32_t* const gcd = w.gcd;
        for (int g = threadIdx.x; g < ng; g += HS_NT) {
            const unsigned long long cg = g == jc ? (unsigned long long)(sc + 1) : gc[g];
            inc[g] = cg * f_units(gt[g], 52);
        }
        __syncthreads();
        const unsigned long long Dn = hs_scan_u64(inc, ng, wtot);
        if (Dn >= (1ull << 53)) return false;
        const double D = (double)Dn * 0x1p-52;
        const double u = row_u(a, row, p);
        // cumulative weights w = p / D over the first n_keep - 1 survivors
        // (the last survivor's is 1.0)
        for (int g = threadIdx.x; g < ng; g += HS_NT) {
            wd[g] = __ddiv_rn((double)gt[g], D);
            gcd[g] = g == jc ? (uint32_t)sc : gc[g];
        }
        __syncthreads();
        for (int g = threadIdx.x; g < ng; g += HS_NT) inc2[g] = (u128)gcd[g] * d_units(wd[g]);
        __syncthreads();
        hs_scan_u128(inc2, ng, wtot2);
        for (int g = threadIdx.x; g < ng; g += HS_NT) sC[g] = g == 0 ? 0.0 : units_d(inc2[g]);
        __syncthreads();
        if (!hs_walk_d(ng, gcd, wd, sC, inc2, stp, u, wtot2, &hm, &o.it_d)) return false;
        int fd = G;
        for (int g = threadIdx.x; g < ng; g += HS_NT)
            if ((uint32_t)stp[g] < gcd[g]) fd = min(fd, g);
        fd = block_min_int(fd, m);
        pos = fd < ng ? (long long)pref[fd] + stp[fd] : n_keep - 1;
    }
    QS_TMARK(row, 7, true);
    // the group holding sorted position pos: the last group starting at or
    // before it
    int lo = 0, hi = G;
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if ((long long)pref[mid] <= pos) lo = mid;
        else hi = mid;
    }
    o.S1 = S1;
    o.S2 = S2;
    o.n_keep = n_keep;
    o.pos = pos;
    o.gp = lo;
    o.jc = jc;
    o.prob = gt[lo];
    return true;
}

// Hands the row to the cluster kernel (thread 0; the caller then leaves the row).
__device__ __forceinline__ void hs_bail(const QsLaunch& a, int row) {
    if (threadIdx.x == 0) a.bail_rows[atomicAdd(a.bail_ctr, 1)] = row;
}

__global__ void __launch_bounds__(HS_NT, 1) qs_hist_kernel(QsLaunch a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const HsLayout L = hs_layout();
    unsigned char* const H = smem_raw + L.off_hist;
    uint32_t* hist = (uint32_t*)H;  // two u16 counts per word (key k: word k/2, half k%2)
    float* gx = (float*)(smem_raw + L.off_gx);
    uint32_t* gc = (uint32_t*)(smem_raw + L.off_gc);
    float* gt = (float*)(smem_raw + L.off_gt);
    int32_t* hid = (int32_t*)(smem_raw + L.off_hid);
    int32_t* hcnt = (int32_t*)(smem_raw + L.off_hcnt);
    float* wx = (float*)(smem_raw + L.off_wx);
    int32_t* wid = (int32_t*)(smem_raw + L.off_wid);
    uint64_t* exp32 = (uint64_t*)(smem_raw + L.off_exp);
    Misc* m = (Misc*)(smem_raw + L.off_misc);
    unsigned long long* pref = (unsigned long long*)(H + HO_PREF);
    unsigned long long* wk = (unsigned long long*)(H + HO_WK);
    unsigned long long* wks = (unsigned long long*)(H + HO_INC);  // the window's keys sorted (until the sums)
    int* wm = (int*)(H + HO_WM);
    __shared__ HsMisc hm;
    __shared__ unsigned long long wtot[NWARPS];
    __shared__ int hs_wc[NWARPS];  // matches per warp (the drawn element's search)
    __shared__ u128 wtot2[NWARPS];
    if (threadIdx.x < 32) exp32[threadIdx.x] = qs_tab_exp32_d[threadIdx.x];
    const float NEG_INF = -__int_as_float(0x7f800000);
    const float POS_INF = __int_as_float(0x7f800000);
    const int V = a.V;
    __syncthreads();

    for (int ri = blockIdx.x; ri < a.hs_nrows;) {
        const int row = a.hs_rows[ri];
        if (threadIdx.x == 0) {
            m->prm = a.params[row];
            hm.bail = 0;
            hm.nuniq = 0;
            hm.found_id = -1;
            hm.nwm = 0;
        }
        __syncthreads();
        const bool arrived = wait_ready(a, row);
        const qsamp_row_params& p = m->prm;
        RowCtx r;
        r.p = &m->prm;
        r.row = row;
        r.V = V;
        r.lo = 0;
        r.hi = V;
        r.len = V;
        r.rowp = (const char*)a.logits + (size_t)row * (size_t)a.row_stride * 2;
        r.dtype = QSAMP_BF16;
        r.cap = p.softcap;
        r.cap_on = p.softcap > 0.0f;
        r.T = p.temperature;
        r.div_on = p.temperature > 0.0f && p.temperature != 1.0f;
        r.force_on = false;
        r.force = -1;
        r.mask = a.masks ? a.masks + (size_t)row * (size_t)a.mask_stride : nullptr;
        r.lut = nullptr;
        if (r.cap_on && a.luts)
            for (int q = 0; q < MAX_LUT; ++q)
                if (a.lut_caps[q] == p.softcap) r.lut = a.luts + (size_t)q * 65536;
        const uint16_t* rp = (const uint16_t*)r.rowp;
        const bool rep_on = p.repetition_penalty != 1.0f;
        const bool fp_on = p.frequency_penalty != 0.0f || p.presence_penalty != 0.0f;
        if (!arrived) {
            if (threadIdx.x == 0) write_skipped(a, row);
            goto next_row;
        }
        {
            QS_TMARK(row, 0, true);
            // ---- 1. the penalty window: distinct ids with their counts
            for (int q = threadIdx.x; q < 65536 / 8; q += HS_NT) ((uint4*)hist)[q] = make_uint4(0u, 0u, 0u, 0u);
            hs_window(a, row, p, V, hid, hcnt, wid, hm);
            if (hm.bail) {
                hs_bail(a, row);
                goto next_row;
            }
            const int nuniq = hm.nuniq;
            QS_TMARK(row, 1, true);

            // ---- 2. the row, once: allow-mask and histogram by key
            int ninf = 0;
            const int nvec = a.vec_ok ? V / 8 : 0;
            for (int g0 = threadIdx.x; g0 < nvec; g0 += HS_LD * HS_NT) {
                uint4 q[HS_LD];
#pragma unroll
                for (int u = 0; u < HS_LD; ++u) {
                    const int g = g0 + u * HS_NT;
                    q[u] = g < nvec ? __ldg((const uint4*)(rp + 8 * g)) : make_uint4(0u, 0u, 0u, 0u);
                }
#pragma unroll
                for (int u = 0; u < HS_LD; ++u) {
                    const int g = g0 + u * HS_NT;
                    if (g < nvec) {
                        const int i0 = 8 * g;
                        const uint32_t mw = r.mask ? (r.mask[i0 >> 5] >> (i0 & 31)) : 0xffu;
                        const uint32_t w4[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            if (!((mw >> e) & 1u)) {
                                ++ninf;
                            } else {
                                const uint32_t k = hs_key((w4[e >> 1] >> ((e & 1) * 16)) & 0xffffu);
                                atomicAdd(&hist[k >> 1], 1u << ((k & 1u) << 4));
                            }
                        }
                    }
                }
            }
            for (int i = 8 * nvec + threadIdx.x; i < V; i += HS_NT) {
                if (r.mask && !((r.mask[i >> 5] >> (i & 31)) & 1u)) {
                    ++ninf;
                } else {
                    const uint32_t k = hs_key(rp[i]);
                    atomicAdd(&hist[k >> 1], 1u << ((k & 1u) << 4));
                }
            }
            ninf = block_sum_int(ninf, m);  // (its barriers complete the histogram)
            QS_TMARK(row, 2, true);

            // ---- 3. the total (an overflowed bin only lowers it), NaN and
            // infinite patterns, the largest counted key
            {
                unsigned long long tot = 0;
                int special = 0, top = -1;
                for (int q = threadIdx.x; q < 32768; q += HS_NT) {
                    const uint32_t wv = hist[q];
                    tot += (wv & 0xffffu) + (wv >> 16);
                    if (wv && (q < HS_KLO / 2 || q >= HS_KHI / 2)) special = 1;
                    if (wv) top = max(top, (wv >> 16) ? 2 * q + 1 : 2 * q);
                }
                for (int o = 16; o > 0; o >>= 1) {
                    tot += __shfl_down_sync(FULLMASK, tot, o);
                    special |= __shfl_down_sync(FULLMASK, special, o);
                    top = max(top, __shfl_down_sync(FULLMASK, top, o));
                }
                if ((threadIdx.x & 31) == 0) {
                    m->red_u[threadIdx.x >> 5] = tot;
                    m->red_i[threadIdx.x >> 5] = special;
                    m->red_u2[threadIdx.x >> 5] = (unsigned long long)(long long)top;
                }
                __syncthreads();
                if (threadIdx.x == 0) {
                    unsigned long long T = 0;
                    int sp = 0;
                    long long tp = -1;
                    for (int w = 0; w < NWARPS; ++w) {
                        T += m->red_u[w];
                        sp |= m->red_i[w];
                        tp = max(tp, (long long)m->red_u2[w]);
                    }
                    hm.top_key = (int)tp;
                    if (T != (unsigned long long)(V - ninf) || sp) hm.bail = 2;
                }
                __syncthreads();
            }
            if (hm.bail) {
                hs_bail(a, row);
                goto next_row;
            }
            // the window's elements: penalised values (sampling.cpp:124-135
            // plus frequency / presence); allowed ones leave the histogram
            float wmax = NEG_INF;
            for (int u = threadIdx.x; u < nuniq; u += HS_NT) {
                const int id = wid[u];
                const uint32_t bits = rp[id];
                const bool allowed = !r.mask || ((r.mask[id >> 5] >> (id & 31)) & 1u);
                uint32_t slot = ((uint32_t)id * 2654435761u) & (HS_HT - 1);
                while (hid[slot] != id) slot = (slot + 1) & (HS_HT - 1);
                const int c = hcnt[slot];
                float v = qs_bf16_to_f32((uint16_t)bits);
                if (r.cap_on) v = r.lut ? r.lut[bits] : qs_softcap(v, r.cap);
                if (!allowed) v = NEG_INF;
                if (rep_on) v = v < 0.0f ? __fmul_rn(v, p.repetition_penalty) : __fdiv_rn(v, p.repetition_penalty);
                if (fp_on) {
                    v = __fsub_rn(v, __fmul_rn((float)c, p.frequency_penalty));
                    v = __fsub_rn(v, p.presence_penalty);
                }
                v = post_value(r, v);
                wx[u] = v;
                if (allowed) {
                    const uint32_t k = hs_key(bits);
                    atomicSub(&hist[k >> 1], 1u << ((k & 1u) << 4));
                }
                wmax = fmaxf(wmax, v);
            }
            // ---- 4. the row max
            for (int o = 16; o > 0; o >>= 1) wmax = fmaxf(wmax, __shfl_down_sync(FULLMASK, wmax, o));
            if ((threadIdx.x & 31) == 0) m->red_f[threadIdx.x >> 5] = wmax;
            __syncthreads();
            if (threadIdx.x == 0) {
                float wmx = NEG_INF;
                for (int w = 0; w < NWARPS; ++w) wmx = fmaxf(wmx, m->red_f[w]);
                int k = hm.top_key;  // (it may have lost its only elements to the window)
                while (k >= HS_KLO && hs_count(hist, k) == 0u) --k;
                const float xt = k >= HS_KLO ? hs_value(r, (uint32_t)k) : NEG_INF;
                const float M = fmaxf(xt, wmx);
                hm.M = M;
                if (!(M > NEG_INF) || !(M < POS_INF)) hm.bail = 3;
            }
            __syncthreads();
            if (hm.bail) {
                hs_bail(a, row);
                goto next_row;
            }
            const float M = hm.M;
            QS_TMARK(row, 3, true);

            // ---- 5. groups: counted keys with x - M >= HS_DMIN, descending.
            // The key -> value map is monotone, so those keys are the range
            // [kmin, top key]: kmin by a 32-way search of warp 0, then the
            // range split evenly, highest keys first, over the threads.
            if (threadIdx.x < 32) {
                const int lane = threadIdx.x;
                auto near = [&](int k) { return __fsub_rn(hs_value(r, (uint32_t)k), M) >= HS_DMIN; };
                int lo = HS_KLO, hi = HS_KHI;  // the smallest k with near(k) is in [lo, hi] (hi: none)
                while (hi - lo > 32) {
                    const int pt = lo + (int)(((long long)(hi - lo) * (lane + 1)) / 32);  // lane 31: hi
                    const bool t = pt < hi && near(pt);
                    const uint32_t bt = __ballot_sync(FULLMASK, t) | 0x80000000u;
                    const int f = __ffs(bt) - 1;  // first point at which near holds (31: hi)
                    const int pf = lo + (int)(((long long)(hi - lo) * (f + 1)) / 32);
                    const int pp = f > 0 ? lo + (int)(((long long)(hi - lo) * f) / 32) + 1 : lo;
                    lo = pp;
                    hi = pf;
                }
                const int kk = lo + lane;
                const bool t = kk < hi && near(kk);
                const uint32_t bt = __ballot_sync(FULLMASK, t);
                if (lane == 0) hm.kmin = bt ? lo + __ffs(bt) - 1 : hi;
            }
            __syncthreads();
            QS_TMARK(row, 15, true);
            const int kmin = hm.kmin;
            const int ktop = hm.top_key;
            const int nkeys = ktop >= kmin ? ktop - kmin + 1 : 0;
            const int per = (nkeys + HS_NT - 1) / HS_NT;
            const int khi_t = ktop - per * (int)threadIdx.x;          // this thread: keys (klo_t, khi_t], descending
            const int klo_t = max(kmin - 1, khi_t - per);
            int mine = 0;
            for (int k = khi_t; k > klo_t; --k)
                if (hs_count(hist, k)) ++mine;
            int npg = 0;
            const int off = block_excl_scan_int(mine, npg, m);
            if (npg + nuniq > HS_GMAX) {
                hs_bail(a, row);
                goto next_row;
            }
            {
                // the keys first (the non-empty ones crowd into a few threads'
                // ranges), their values after, spread over every thread
                int at = off;
                for (int k = khi_t; k > klo_t; --k) {
                    const uint32_t c = hs_count(hist, k);
                    if (!c) continue;
                    gx[at] = __int_as_float(k);
                    gc[at] = c;
                    ++at;
                }
            }
            __syncthreads();  // (the histogram is read no more)
            for (int g = threadIdx.x; g < npg; g += HS_NT) gx[g] = hs_value(r, (uint32_t)__float_as_int(gx[g]));
            QS_TMARK(row, 16, true);
            int nw = 0;
            {
                int mw = 0;
                for (int u = threadIdx.x; u < nuniq; u += HS_NT)
                    if (wx[u] > NEG_INF && __fsub_rn(wx[u], M) >= HS_DMIN) ++mw;
                int o2 = block_excl_scan_int(mw, nw, m);
                for (int u = threadIdx.x; u < nuniq; u += HS_NT)
                    if (wx[u] > NEG_INF && __fsub_rn(wx[u], M) >= HS_DMIN)
                        wk[o2++] = ((unsigned long long)qs_key(wx[u]) << 32) | (uint32_t)u;
                __syncthreads();
                // descending order by counting (the keys are distinct: the low
                // word is the entry's index); every thread reads the same key
                // at a time (a shared-memory broadcast)
                for (int j = threadIdx.x; j < nw; j += HS_NT) {
                    const unsigned long long kj = wk[j];
                    int rk = 0;
                    for (int i = 0; i < nw; ++i) rk += wk[i] > kj;
                    wks[rk] = kj;
                }
                __syncthreads();
            }
            const int G = npg + nw;
            QS_TMARK(row, 4, true);
            // merge: pattern group i goes to i + #{window values > x_i},
            // window element j to j + #{pattern groups with value >= its value}
            {
                float px[HS_GPT];
                uint32_t pc[HS_GPT];
                int pd[HS_GPT];
#pragma unroll
                for (int e = 0; e < HS_GPT; ++e) {
                    const int i = threadIdx.x * HS_GPT + e;
                    pd[e] = -1;
                    px[e] = 0.0f;
                    pc[e] = 0u;
                    if (i < npg) {
                        px[e] = gx[i];
                        pc[e] = gc[i];
                        int lo = 0, hi = nw;  // first window entry with value <= px
                        while (lo < hi) {
                            const int mid = (lo + hi) >> 1;
                            if (qs_unkey((uint32_t)(wks[mid] >> 32)) > px[e]) lo = mid + 1;
                            else hi = mid;
                        }
                        pd[e] = i + lo;
                    }
                }
                float wv[HS_WMAX / HS_NT];
                int wdst[HS_WMAX / HS_NT];
#pragma unroll
                for (int e = 0; e < HS_WMAX / HS_NT; ++e) {
                    const int j = threadIdx.x + e * HS_NT;
                    wdst[e] = -1;
                    wv[e] = 0.0f;
                    if (j < nw) {
                        wv[e] = qs_unkey((uint32_t)(wks[j] >> 32));
                        int lo = 0, hi = npg;  // first pattern group with value < wv
                        while (lo < hi) {
                            const int mid = (lo + hi) >> 1;
                            if (gx[mid] >= wv[e]) lo = mid + 1;
                            else hi = mid;
                        }
                        wdst[e] = j + lo;
                    }
                }
                __syncthreads();
#pragma unroll
                for (int e = 0; e < HS_GPT; ++e)
                    if (pd[e] >= 0) {
                        gx[pd[e]] = px[e];
                        gc[pd[e]] = pc[e];
                    }
#pragma unroll
                for (int e = 0; e < HS_WMAX / HS_NT; ++e)
                    if (wdst[e] >= 0) {
                        gx[wdst[e]] = wv[e];
                        gc[wdst[e]] = 1u;
                    }
                __syncthreads();
            }
            QS_TMARK(row, 17, true);
            // group start positions in the sorted row
            for (int g = threadIdx.x; g < G; g += HS_NT) pref[g] = gc[g];
            __syncthreads();
            hs_scan_u64(pref, G, wtot);

            QS_TMARK(row, 18, true);
            // ---- 6. the sums and the draw over the groups
            HsDrawn dr;
            if (!hs_sums_draw(a, row, p, G, gx, gc, gt, hs_arrays(H), exp32, M, hm, wtot, wtot2, m, dr)) {
                hs_bail(a, row);
                goto next_row;
            }
            const float S1 = dr.S1, S2 = dr.S2, prob = dr.prob;
            const long long n_keep = dr.n_keep, pos = dr.pos;
            const int gp = dr.gp;
            // ---- 7. the element at sorted position pos: the first group of
            // its value, its rank among the row's elements of that value
            // (ascending id), and the element of that rank
            const float xs = gx[gp];
            int glo = gp;
            while (glo > 0 && gx[glo - 1] == xs) --glo;
            const long long rank = pos - (long long)pref[glo];
            // the row's elements of value xs (the groups of that value): the
            // search below counts from the nearer end of the row
            int ghi = gp;
            while (ghi + 1 < G && gx[ghi + 1] == xs) ++ghi;
            const long long n_xs = (ghi + 1 < G ? (long long)pref[ghi + 1] : (long long)pref[ghi] + gc[ghi]) -
                                   (long long)pref[glo];
            const bool from_end = 2 * rank >= n_xs;
            const long long target = from_end ? n_xs - 1 - rank : rank;
            // the keys whose (non-window) elements have value xs: [klo, khi]
            // (the key -> value map is monotone: two 32-way searches, one warp each)
            if (threadIdx.x < 32)
                hm.klo = hs_warp_search(HS_KLO, HS_KHI, [&](int k) { return hs_value(r, (uint32_t)k) >= xs; });
            else if (threadIdx.x < 64)
                hm.khi = hs_warp_search(HS_KLO, HS_KHI, [&](int k) { return hs_value(r, (uint32_t)k) > xs; }) - 1;
            __syncthreads();
            const int klo = hm.klo, khi = hm.khi;
            // the window's elements of value xs (allowed ones: -inf never equals xs)
            for (int u = threadIdx.x; u < nuniq; u += HS_NT)
                if (wx[u] == xs) wm[atomicAdd(&hm.nwm, 1)] = wid[u];
            __syncthreads();
            const int nwm = hm.nwm;
            QS_TMARK(row, 10, true);
            // the 8 elements from i0 (a multiple of 8) that hold value xs:
            // keys [klo, khi] outside the window and allowed, and the window's
            // elements of that value; ld8 loads them, flags_of tests them
            auto ld8 = [&](int i0) -> uint4 {
                if (i0 >= V) return make_uint4(0u, 0u, 0u, 0u);
                if (a.vec_ok && i0 + 8 <= V) return __ldg((const uint4*)(rp + i0));
                uint32_t w[4] = {0u, 0u, 0u, 0u};
                for (int e = 0; e < 8; ++e)
                    if (i0 + e < V) w[e >> 1] |= (uint32_t)rp[i0 + e] << ((e & 1) * 16);
                return make_uint4(w[0], w[1], w[2], w[3]);
            };
            auto flags_of = [&](int i0, uint4 q) -> uint32_t {
                uint32_t flags = 0;
                if (i0 >= V) return 0u;
                const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const int i = i0 + e;
                    const int k = (int)hs_key((w4[e >> 1] >> ((e & 1) * 16)) & 0xffffu);
                    if (i >= V || k < klo || k > khi) continue;
                    if (r.mask && !((r.mask[i >> 5] >> (i & 31)) & 1u)) continue;
                    bool inwin = false;
                    if (nuniq) {
                        uint32_t slot = ((uint32_t)i * 2654435761u) & (HS_HT - 1);
                        while (hid[slot] != -1) {
                            if (hid[slot] == i) {
                                inwin = true;
                                break;
                            }
                            slot = (slot + 1) & (HS_HT - 1);
                        }
                    }
                    if (!inwin) flags |= 1u << e;
                }
                for (int u = 0; u < nwm; ++u) {
                    const int d = wm[u] - i0;
                    if (d >= 0 && d < 8) flags |= 1u << d;
                }
                return flags;
            };
            // the rank-th of them in id order, in super-chunks of 16 x 1024
            // elements: warp w counts elements [s + 1024 w, s + 1024 (w + 1))
            // in four 256-element pieces (their loads in flight together); one
            // prefix over the warps tells whether the rank-th lies in this
            // super-chunk, and which warp and piece hold it. Super-chunks are
            // taken from the end of the row down when the rank-th is nearer
            // the end (target counts from there; inside the super-chunk that
            // holds it the rank is counted forward again).
            {
                const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
                const int nsc = (V + NWARPS * 1024 - 1) / (NWARPS * 1024);
                long long acc = 0;
                for (int q = 0; q < nsc; ++q) {
                    const int sc = (from_end ? nsc - 1 - q : q) * (NWARPS * 1024);
                    const int wb = sc + warp * 1024;
                    uint4 qv[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) qv[u] = ld8(wb + u * 256 + 8 * lane);
                    uint32_t fl[4];
                    int pc[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        fl[u] = flags_of(wb + u * 256 + 8 * lane, qv[u]);
                        int cn = __popc(fl[u]);
                        for (int o = 16; o > 0; o >>= 1) cn += __shfl_xor_sync(FULLMASK, cn, o);
                        pc[u] = cn;
                    }
                    if (lane == 0) hs_wc[warp] = pc[0] + pc[1] + pc[2] + pc[3];
                    __syncthreads();
                    int before = 0, tot = 0;  // (within the super-chunk)
                    for (int w2 = 0; w2 < NWARPS; ++w2) {
                        if (w2 < warp) before += hs_wc[w2];
                        tot += hs_wc[w2];
                    }
                    __syncthreads();  // (hs_wc is rewritten by the next super-chunk)
                    if (acc + tot > target) {
                        // the forward rank inside this super-chunk
                        const int lr = from_end ? (int)(tot - 1 - (target - acc)) : (int)(target - acc);
                        const int wc = pc[0] + pc[1] + pc[2] + pc[3];
                        if (lr >= before && lr < before + wc) {
                            int want = lr - before;
                            int u = 0;
                            while (u < 3 && want >= pc[u]) want -= pc[u++];
                            uint32_t f = fl[0];
#pragma unroll
                            for (int j = 1; j < 4; ++j)
                                if (u == j) f = fl[j];
                            const int nm = __popc(f);
                            int incl = nm;
                            for (int o = 1; o < 32; o <<= 1) {
                                const int v = __shfl_up_sync(FULLMASK, incl, o);
                                if (lane >= o) incl += v;
                            }
                            if (want >= incl - nm && want < incl) {
                                int left = want - (incl - nm);
                                for (int e = 0; e < 8; ++e)
                                    if ((f >> e) & 1u) {
                                        if (left == 0) {
                                            hm.found_id = wb + u * 256 + 8 * lane + e;
                                            break;
                                        }
                                        --left;
                                    }
                            }
                        }
                        break;  // (uniform: every thread saw the same totals)
                    }
                    acc += tot;
                }
            }
            __syncthreads();
            QS_TMARK(row, 8, true);
            QS_NOTE(row, 9, G, true);
            QS_NOTE(row, 11, dr.it_s, true);
            QS_NOTE(row, 12, dr.it_c, true);
            QS_NOTE(row, 13, dr.it_d, true);
            QS_NOTE(row, 14, dr.jc + 1, true);
            if (hm.found_id < 0) {  // (not expected: the groups count these elements)
                hs_bail(a, row);
                goto next_row;
            }
            if (threadIdx.x == 0) {
                qsamp_row_result res;
                res.token = hm.found_id;
                res.position = (int)pos;
                res.n_keep = (int)n_keep;
                res.drew = n_keep >= 2 ? 1 : 0;
                res.sum_exp = S1;
                res.sum_keep = S2;
                res.max_logit = M;
                res.prob = prob;
                write_result(a, row, res);
            }
        }
    next_row:
        __syncthreads();
        if (threadIdx.x == 0) hm.next_ri = (int)gridDim.x + atomicAdd(a.hs_ctr, 1);
        __syncthreads();
        ri = hm.next_ri;
    }
}
