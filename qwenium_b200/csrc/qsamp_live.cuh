// qsamp_live.cuh -- the live-list path for fp32 full-vocabulary rows
// (included by qsamp_kernels.cu inside namespace qs, after qsamp_hist.cuh).
//
// An element x of a row can change none of the reference's float sums once
// expf(x - M) < 2^-25 (x - M < HS_DMIN): the sums start at expf(0) = 1 and
// every later term of that size is lost in the rounding (sampling.cpp:171,
// :173-178, :184-188). When a row holds at most HS_GMAX elements within
// HS_DMIN of its maximum -- a peaked row: a low temperature, a confident
// model -- those LIVE elements, sorted as the reference sorts them
// (sampling.cpp:158-163: value descending, equal values by ascending id),
// carry every sum, the top-p cut and the draw, and the histogram path's
// group walks (hs_sums_draw) finish the row exactly. One CTA (512 threads)
// per row:
//   1. the penalty window (ids with counts, and a bit per vocabulary id);
//   2. the row from HBM: allow-mask, soft-cap, /T, the row max M;
//   3. the row again (from L2): the live elements' composite keys (value,
//      id) into shared memory; more than HS_GMAX of them return the row;
//   4. a bitonic sort of the keys, the groups of equal values and their
//      start positions, the sorted ids;
//   5. the sums and the draw over the groups; the drawn sorted position's
//      id is read off the sorted ids (no third pass over the row).
//
// Rows are shared with the cluster kernel, which runs at the same time: the
// host lists the candidate rows by falling temperature (a flatter row has
// more live elements); the cluster kernel claims from the front of the
// list, this kernel from the back, one claim word per row. A row this path
// cannot serve (too many live elements, an infinite value, a sum the group
// walks do not prove exact) goes to a return list that the cluster kernel
// serves while it runs, and a second cluster launch after both kernels
// serves what is left; no kernel waits for the other.

constexpr int LV_VMAX = 262144;  // vocabulary served (the window's id bits fit shared memory)

struct LvLayout {
    int off_h, off_gx, off_gc, off_gt, off_sid, off_wx, off_wid, off_exp, off_misc, total;
};
// The window's id bits and hash table live in the groups' area until the
// second pass is done; the key list in the walks' area until the groups are
// built.
__host__ __device__ inline LvLayout lv_layout() {
    LvLayout L;
    int o = 0;
    L.off_h = o;   o = align_up(o + 131072, 16);             // keys u64[GMAX], then the walks' arrays
    L.off_gx = o;  o = align_up(o + HS_GMAX * 4, 16);        // group value | window id bits (32 KB)
    L.off_gc = o;  o = align_up(o + HS_GMAX * 4, 16);        // group count |
    L.off_gt = o;  o = align_up(o + HS_GMAX * 4, 16);        // group term  | window hash ids, counts
    L.off_sid = o; o = align_up(o + HS_GMAX * 4, 16);        // ids in sorted order
    L.off_wx = o;  o = align_up(o + HS_WMAX * 4, 16);        // distinct window ids' values
    L.off_wid = o; o = align_up(o + HS_WMAX * 4, 16);        //   and ids
    L.off_exp = o; o = align_up(o + 32 * 8, 16);
    L.off_misc = o; o = align_up(o + (int)sizeof(Misc), 16);
    L.total = o;
    return L;
}
static_assert(LV_VMAX / 8 + 2 * HS_HT * 4 <= 3 * HS_GMAX * 4, "window bits and hash fit the groups' area");
static_assert(HS_GMAX * 8 <= HO_PREF, "the key list stays clear of the group starts");

// This kernel's next candidate row (one thread): the back of the list.
__device__ int lv_claim_back(const QsLaunch& a) {
    const int j = atomicAdd(&a.lv_q[1], 1);
    const int i = a.lv_n - 1 - j;
    if (i < 0 || atomicCAS(&a.lv_taken[i], 0, 1) != 0) return -1;
    return a.lv_rows[i];
}
__device__ void lv_return(const QsLaunch& a, int row) {
    if (threadIdx.x == 0) {
        const int k = atomicAdd(&a.lv_q[2], 1);
        atomicExch(&a.lv_ret[k], row + 1);
    }
}

__global__ void __launch_bounds__(HS_NT, 1) qs_live_kernel(QsLaunch a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const LvLayout L = lv_layout();
    unsigned char* const H = smem_raw + L.off_h;
    unsigned long long* keys = (unsigned long long*)H;
    float* gx = (float*)(smem_raw + L.off_gx);
    uint32_t* gc = (uint32_t*)(smem_raw + L.off_gc);
    float* gt = (float*)(smem_raw + L.off_gt);
    uint32_t* wbits = (uint32_t*)(smem_raw + L.off_gx);
    int32_t* hid = (int32_t*)(smem_raw + L.off_gx + LV_VMAX / 8);
    int32_t* hcnt = hid + HS_HT;
    uint32_t* sid = (uint32_t*)(smem_raw + L.off_sid);
    float* wx = (float*)(smem_raw + L.off_wx);
    int32_t* wid = (int32_t*)(smem_raw + L.off_wid);
    uint64_t* exp32 = (uint64_t*)(smem_raw + L.off_exp);
    Misc* m = (Misc*)(smem_raw + L.off_misc);
    const HsArrays w = hs_arrays(H);
    __shared__ HsMisc hm;
    __shared__ unsigned long long wtot[NWARPS];
    __shared__ u128 wtot2[NWARPS];
    __shared__ int lv_n, lv_row, lv_special;
    if (threadIdx.x < 32) exp32[threadIdx.x] = qs_tab_exp32_d[threadIdx.x];
    const float NEG_INF = -__int_as_float(0x7f800000);
    const float POS_INF = __int_as_float(0x7f800000);
    const int V = a.V;
    const int nw32 = (V + 31) / 32;
    if (threadIdx.x == 0) lv_row = lv_claim_back(a);
    __syncthreads();

    while (lv_row >= 0) {
        const int row = lv_row;
        if (threadIdx.x == 0) {
            m->prm = a.params[row];
            hm.bail = 0;
            hm.nuniq = 0;
            lv_n = 0;
            lv_special = 0;
        }
        for (int q = threadIdx.x; q < nw32; q += HS_NT) wbits[q] = 0u;
        __syncthreads();
        const qsamp_row_params& p = m->prm;
        RowCtx r;
        r.p = &m->prm;
        r.row = row;
        r.V = V;
        r.lo = 0;
        r.hi = V;
        r.len = V;
        r.rowp = (const char*)a.logits + (size_t)row * (size_t)a.row_stride * 4;
        r.dtype = QSAMP_F32;
        r.cap = p.softcap;
        r.cap_on = p.softcap > 0.0f;
        r.T = p.temperature;
        r.div_on = p.temperature > 0.0f && p.temperature != 1.0f;
        r.force_on = false;
        r.force = -1;
        r.mask = a.masks ? a.masks + (size_t)row * (size_t)a.mask_stride : nullptr;
        r.lut = nullptr;
        const float* rp = (const float*)r.rowp;
        // the value of a non-window element (soft-cap, allow-mask, /T, canon)
        auto value_of = [&](int i, float raw, bool allowed) -> float {
            float v = raw;
            if (r.cap_on) v = qs_softcap(raw, r.cap);
            if (!allowed) v = NEG_INF;
            return post_value(r, v);
        };
        QS_TMARK(row, 0, true);
        {
            // ---- 1. the penalty window: ids with counts, and their bits
            hs_window(a, row, p, V, hid, hcnt, wid, hm);
            if (hm.bail) {
                lv_return(a, row);
                goto next_row;
            }
            const int nuniq = hm.nuniq;
            for (int u = threadIdx.x; u < nuniq; u += HS_NT) atomicOr(&wbits[wid[u] >> 5], 1u << (wid[u] & 31));
            float wmax = NEG_INF;
            for (int u = threadIdx.x; u < nuniq; u += HS_NT) {
                const int id = wid[u];
                const bool allowed = !r.mask || ((r.mask[id >> 5] >> (id & 31)) & 1u);
                float v = rp[id];
                if (r.cap_on) v = qs_softcap(v, r.cap);
                if (!allowed) v = NEG_INF;
                v = hs_penalise(r, p, v, hs_window_count(hid, hcnt, id));
                wx[u] = v;
                wmax = fmaxf(wmax, v);
            }
            __syncthreads();
            QS_TMARK(row, 1, true);

            // ---- 2. the row max (the window's values included)
            const int nvec = a.vec_ok ? V / 8 : 0;
            float bm = wmax;
            int special = wmax == POS_INF;
            for (int b0 = 0; b0 < nvec; b0 += 2 * HS_NT) {
                float4 q[4];
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int g = b0 + u * HS_NT + threadIdx.x;
                    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
                    q[2 * u] = g < nvec ? __ldg((const float4*)(rp + 8 * g)) : z;
                    q[2 * u + 1] = g < nvec ? __ldg((const float4*)(rp + 8 * g + 4)) : z;
                }
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int g = b0 + u * HS_NT + threadIdx.x;
                    if (g >= nvec) continue;
                    const int i0 = 8 * g;
                    const uint32_t mw = r.mask ? (r.mask[i0 >> 5] >> (i0 & 31)) : 0xffu;
                    const uint32_t wb = nuniq ? (wbits[i0 >> 5] >> (i0 & 31)) : 0u;
                    const float xs[8] = {q[2 * u].x, q[2 * u].y, q[2 * u].z, q[2 * u].w,
                                         q[2 * u + 1].x, q[2 * u + 1].y, q[2 * u + 1].z, q[2 * u + 1].w};
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        if ((wb >> e) & 1u) continue;
                        const float x = value_of(i0 + e, xs[e], (mw >> e) & 1u);
                        special |= x == POS_INF;
                        bm = fmaxf(bm, x);
                    }
                }
            }
            for (int i = 8 * nvec + threadIdx.x; i < V; i += HS_NT) {
                if (nuniq && ((wbits[i >> 5] >> (i & 31)) & 1u)) continue;
                const bool allowed = !r.mask || ((r.mask[i >> 5] >> (i & 31)) & 1u);
                const float x = value_of(i, rp[i], allowed);
                special |= x == POS_INF;
                bm = fmaxf(bm, x);
            }
            for (int o = 16; o > 0; o >>= 1) {
                bm = fmaxf(bm, __shfl_down_sync(FULLMASK, bm, o));
                special |= __shfl_down_sync(FULLMASK, special, o);
            }
            if ((threadIdx.x & 31) == 0) {
                m->red_f[threadIdx.x >> 5] = bm;
                if (special) lv_special = 1;
            }
            __syncthreads();
            if (threadIdx.x == 0) {
                float M = NEG_INF;
                for (int q = 0; q < NWARPS; ++q) M = fmaxf(M, m->red_f[q]);
                hm.M = M;
                if (lv_special || !(M > NEG_INF)) hm.bail = 2;
                else if (a.lv_return_all) hm.bail = 4;  // (tests: the row is returned after step 3)
            }
            __syncthreads();
            if (hm.bail == 2) {
                lv_return(a, row);
                goto next_row;
            }
            const float M = hm.M;
            QS_TMARK(row, 2, true);

            // ---- 3. the live elements' keys (value desc, id asc when sorted)
            const int lane = threadIdx.x & 31;
            for (int b0 = 0; b0 < nvec; b0 += 2 * HS_NT) {
                float4 q[4];
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int g = b0 + u * HS_NT + threadIdx.x;
                    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
                    q[2 * u] = g < nvec ? __ldg((const float4*)(rp + 8 * g)) : z;
                    q[2 * u + 1] = g < nvec ? __ldg((const float4*)(rp + 8 * g + 4)) : z;
                }
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int g = b0 + u * HS_NT + threadIdx.x;
                    const int i0 = 8 * g;
                    uint32_t live = 0u;
                    float xv[8];
                    if (g < nvec) {
                        const uint32_t mw = r.mask ? (r.mask[i0 >> 5] >> (i0 & 31)) : 0xffu;
                        const uint32_t wb = nuniq ? (wbits[i0 >> 5] >> (i0 & 31)) : 0u;
                        const float xs[8] = {q[2 * u].x, q[2 * u].y, q[2 * u].z, q[2 * u].w,
                                             q[2 * u + 1].x, q[2 * u + 1].y, q[2 * u + 1].z, q[2 * u + 1].w};
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            xv[e] = value_of(i0 + e, xs[e], (mw >> e) & 1u);
                            if (!((wb >> e) & 1u) && xv[e] > NEG_INF && __fsub_rn(xv[e], M) >= HS_DMIN)
                                live |= 1u << e;
                        }
                    }
                    // one shared-memory reservation per warp (none when no lane has one)
                    if (__ballot_sync(FULLMASK, live != 0u) == 0u) continue;
                    const int cnt = __popc(live);
                    int incl = cnt;
                    for (int o = 1; o < 32; o <<= 1) {
                        const int y = __shfl_up_sync(FULLMASK, incl, o);
                        if (lane >= o) incl += y;
                    }
                    const int wtotal = __shfl_sync(FULLMASK, incl, 31);
                    int base = 0;
                    if (lane == 31 && wtotal) base = atomicAdd(&lv_n, wtotal);
                    base = __shfl_sync(FULLMASK, base, 31) + incl - cnt;
                    for (int e = 0; e < 8; ++e)
                        if ((live >> e) & 1u) {
                            if (base < HS_GMAX) keys[base] = composite(xv[e], i0 + e);
                            ++base;
                        }
                }
            }
            for (int i = 8 * nvec + threadIdx.x; i < V; i += HS_NT) {
                if (nuniq && ((wbits[i >> 5] >> (i & 31)) & 1u)) continue;
                const bool allowed = !r.mask || ((r.mask[i >> 5] >> (i & 31)) & 1u);
                const float x = value_of(i, rp[i], allowed);
                if (x > NEG_INF && __fsub_rn(x, M) >= HS_DMIN) {
                    const int at = atomicAdd(&lv_n, 1);
                    if (at < HS_GMAX) keys[at] = composite(x, i);
                }
            }
            for (int u = threadIdx.x; u < nuniq; u += HS_NT)
                if (wx[u] > NEG_INF && __fsub_rn(wx[u], M) >= HS_DMIN) {
                    const int at = atomicAdd(&lv_n, 1);
                    if (at < HS_GMAX) keys[at] = composite(wx[u], wid[u]);
                }
            __syncthreads();
            const int n = lv_n;
            if (n > HS_GMAX || n < 1 || hm.bail) {
                lv_return(a, row);
                goto next_row;
            }
            QS_TMARK(row, 3, true);

            // ---- 4. sort; groups of equal values, their starts; sorted ids
            const int P2 = next_pow2(n);
            for (int i = n + threadIdx.x; i < P2; i += HS_NT) keys[i] = 0ull;
            __syncthreads();
            if (P2 > 1) bitonic_desc<128>(keys, P2);
            __syncthreads();
            int G = 0;
            {
                // thread t: sorted positions [t * HS_GPT, (t + 1) * HS_GPT)
                const int i0 = threadIdx.x * HS_GPT;
                int mine = 0;
#pragma unroll
                for (int e = 0; e < HS_GPT; ++e) {
                    const int i = i0 + e;
                    if (i < n && (i == 0 || (keys[i] >> 32) != (keys[i - 1] >> 32))) ++mine;
                }
                int at = block_excl_scan_int(mine, G, m);
#pragma unroll
                for (int e = 0; e < HS_GPT; ++e) {
                    const int i = i0 + e;
                    if (i >= n) break;
                    sid[i] = (uint32_t)comp_idx(keys[i]);
                    if (i == 0 || (keys[i] >> 32) != (keys[i - 1] >> 32)) {
                        gx[at] = comp_val(keys[i]);
                        w.pref[at] = (unsigned long long)i;
                        ++at;
                    }
                }
                __syncthreads();
                for (int g = threadIdx.x; g < G; g += HS_NT)
                    gc[g] = (uint32_t)((g + 1 < G ? w.pref[g + 1] : (unsigned long long)n) - w.pref[g]);
                __syncthreads();
            }
            QS_TMARK(row, 4, true);

            // ---- 5. the sums and the draw; the drawn position's id
            HsDrawn dr;
            if (!hs_sums_draw(a, row, p, G, gx, gc, gt, w, exp32, M, hm, wtot, wtot2, m, dr)) {
                lv_return(a, row);
                goto next_row;
            }
            QS_TMARK(row, 8, true);
            QS_NOTE(row, 9, G, true);
            QS_NOTE(row, 11, dr.it_s, true);
            QS_NOTE(row, 12, dr.it_c, true);
            QS_NOTE(row, 13, dr.it_d, true);
            QS_NOTE(row, 14, dr.jc + 1, true);
            if (threadIdx.x == 0) {
                qsamp_row_result res;
                res.token = (int)sid[dr.pos];
                res.position = (int)dr.pos;
                res.n_keep = (int)dr.n_keep;
                res.drew = dr.n_keep >= 2 ? 1 : 0;
                res.sum_exp = dr.S1;
                res.sum_keep = dr.S2;
                res.max_logit = M;
                res.prob = dr.prob;
                write_result(a, row, res);
                atomicAdd(&a.lv_q[3], 1);
            }
        }
    next_row:
        __syncthreads();
        if (threadIdx.x == 0) lv_row = lv_claim_back(a);
        __syncthreads();
    }
}
