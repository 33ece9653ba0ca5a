// qsamp_device.h -- structures shared by the host API (qsamp_api.cu) and the
// selection kernels (qsamp_kernels.cu). Internal; the public C ABI is
// include/qsamp.h.
#ifndef QSAMP_DEVICE_H
#define QSAMP_DEVICE_H

#include <stdint.h>

#include "../../include/qsamp.h"

namespace qs {

constexpr int NT = 512;            // threads per CTA
constexpr int NWARPS = NT / 32;
constexpr int NB = 2048;           // value bins over x = l - max (bin NB-1 = tail)
constexpr float BIN_R = 112.0f;    // bins per nat: bin(x) = min(NB-1, (int)(-x * BIN_R))
constexpr int HIST_MAX = 4096;     // longest penalty window handled on the device
constexpr int SPEC_CAP = 2048;     // elements gathered in sorted order per round
constexpr int KMAX = 1024;         // largest top-k served by the sorted-candidate path
constexpr int MAX_LUT = 4;         // distinct soft-cap values per call with bf16 tables
constexpr int MAX_CLUSTER = 16;

// Device status codes (first error wins; written with atomicCAS).
enum DevStatus : int {
    DEV_OK = 0,
    DEV_TOPK_TOO_LARGE = 1,        // 0 < k < V with k > KMAX
    DEV_ROUNDS_EXHAUSTED = 2,      // the exact walk needed more gather rounds than allowed
    DEV_INTERNAL = 3,
    DEV_TIMEOUT = 4,               // a bounded wait ran out (the kernel returned early)
};

struct QsLaunch {
    const void* logits;
    int dtype;                     // QSAMP_F32 / QSAMP_BF16
    int B, V;
    long long row_stride;          // elements
    int vec_ok;                    // rows are 16-byte aligned: vector loads allowed
    const qsamp_row_params* params;  // device [B]
    const int32_t* hist;           // device [B][hist_stride] or null
    int hist_stride;
    const int32_t* hist_len;       // device [B] or null
    const uint32_t* masks;         // device or null
    long long mask_stride;         // words per row; 0 = shared
    const double* u;               // device [B] or null (then Philox)
    unsigned long long philox_offset;
    const float* luts;             // device [MAX_LUT][65536]
    float lut_caps[MAX_LUT];       // cap of each table; 0 = empty slot
    qsamp_row_result* results;     // device [B]
    int32_t* out_ids;              // device [B] or null
    int32_t* top_ids;              // device [B][top_cap] or null
    float* top_probs;              // device [B][top_cap] or null
    int top_cap;
    int* status;                   // device word
    int n_s;                       // slice length per CTA (multiple of 8)
    int max_rounds;                // gather rounds allowed per row
    const int32_t* rows;           // rows this launch serves, or null: all B rows
    int nrows;                     // entries of rows
    int* row_ctr;                  // row queue of the cluster kernel (zero at launch), or null
    int* srow_ctr;                 // row queue of the stream kernel (zero at launch), or null
    // vocab-sharded selection: this launch holds logits [v_offset, v_offset + V)
    // of a V_total vocabulary; hist ids and force_token are global ids
    int v_offset;
    int V_total;                   // 0: V (unsharded)
    float* cand_vals;              // non-null: write each row's sorted local top-k here
    int32_t* cand_ids;             //   [B][cand_k] values / global ids (-1: padding)
    int cand_k;
    // rows arrive while the kernels run (host entry point): row r may be read
    // once ready[r / ready_rows] != 0; null: all rows are resident at launch
    const int* ready;
    int ready_rows;
    unsigned long long ready_wait_ns;  // longest wait for one ready flag
    // the cluster kernel serves rows[0 .. nrows + *nrows_dev) when nrows_dev
    // is set (rows handed on by the histogram kernel are appended on the device)
    const int* nrows_dev;
    // the histogram kernel (bf16 full-vocabulary rows): its rows, its queue,
    // and where it appends the rows it hands to the cluster kernel
    const int32_t* hs_rows;
    int hs_nrows;
    int* hs_ctr;
    int32_t* bail_rows;
    int* bail_ctr;
    // fp32 full-vocabulary rows shared by the cluster kernel and the
    // live-list kernel (running at the same time): candidates
    // lv_rows[0, lv_n), highest temperature first. The cluster kernel claims
    // from the front, the live-list kernel from the back (one claim word per
    // candidate); rows the live-list kernel returns (entries row + 1, 0 until
    // written) are served by the cluster kernel and by a second cluster
    // launch after both.
    const int32_t* lv_rows;        // null: no candidates
    int lv_n;
    int* lv_q;                     // [0] front, [1] back, [2] returned rows, [3] rows the live-list kernel served
    int* lv_taken;                 // [lv_n]
    int* lv_ret;                   // [lv_n]
    int* lv_rclaim;                // [lv_n]
    int lv_serve_returns;          // cluster kernel: also serve returned rows
    int lv_return_all;             // live-list kernel (tests): return every row after its passes
};

// Dynamic shared-memory layout; identical on host (sizing) and device.
struct SmemLayout {
    int off_vals, off_cnt, off_tsum, off_ksum, off_tx, off_sstart, off_flag, off_gs, off_gc, off_tie, off_vmin, off_vmax,
        off_vcnt, off_spec, off_spect, off_exp, off_misc, total;
};

// Per-CTA scalars kept at off_misc.
struct __align__(16) Misc {
    qsamp_row_params prm;
    float red_f[NWARPS];
    int red_i[NWARPS];
    unsigned long long red_u[NWARPS];
    unsigned long long red_u2[NWARPS];
    float cmax;            // this CTA's slice max
    int cmax_idx;
    float M;               // row max
    int argmax;
    int cmd;               // command for this CTA (written by CTA 0)
    int spec_n;            // CTA 0: gathered elements this round
    int eq_count;          // elements equal to the selection key in this slice
    int sel_bin;           // broadcast radix bin
    int sel_rem;           // broadcast remaining rank
    int sel_cnt;           // broadcast count of the chosen bin
    int next_ri;           // leading CTA: the cluster's next row-list entry
    int next_row;          //   and the row it names (-1: none left)
    int skip;              // this CTA's row data did not arrive in time (wait ran out)
    int skip_row;          // some CTA of the cluster skips the row: token -1
    unsigned long long sel_remw;  // broadcast remaining weight (weighted select)
    float S_n, S_c;        // exact sums (broadcast)
    int first_round;
    int round;
    int ninf;              // -inf elements in this slice (full path)
    int kmode, kfrom, kto; // integer sums to compute in this pass: 1 = S, 2 = top-p
    int neg_quota;         // lowest-id -inf elements to gather (row total)
    int n_sel;             // survivors cap: min(top_k, V) or V
    int cum_bmax;          // last bin whose cum k-sums are needed
    int tail_mode;         // weighted select restricted to the tail bin
    float tail_x;          // tail threshold on x
    uint32_t sel_prefix, sel_mask;
    uint32_t gather_bits[NB / 32];
};

__host__ __device__ inline int align_up(int x, int a) { return (x + a - 1) / a * a; }

// vcounts: the per-bin counts of the smallest / largest value (bf16 rows,
// whose equal logits fill whole bins); fp32 layouts leave them out.
__host__ __device__ inline SmemLayout smem_layout(int n_s, bool vcounts = true) {
    SmemLayout L;
    int o = 0;
    L.off_vals = o;   o = align_up(o + n_s * 4, 16);
    L.off_cnt = o;    o = align_up(o + NB * 4, 16);
    L.off_tsum = o;   o = align_up(o + NB * 4, 16);     // float prediction sums
    L.off_ksum = o;   o = align_up(o + NB * 8, 16);     // u64 quantised sums
    L.off_tx = o;     o = align_up(o + NB * 8, 16);     // u64 fixed-point exact t sums (2^-40)
    L.off_sstart = o; o = align_up(o + NB * 4, 16);     // float S at bin start
    L.off_flag = o;   o = align_up(o + NB, 16);
    L.off_gs = o;     o = align_up(o + NB, 16);
    L.off_gc = o;     o = align_up(o + NB, 16);
    L.off_tie = o;    o = align_up(o + NB / 8, 16);
    L.off_vmin = o;   o = align_up(o + NB * 4, 16);     // smallest / largest value key per bin:
    L.off_vmax = o;   o = align_up(o + NB * 4, 16);     // equal = every element of the bin has one value
    L.off_vcnt = o;   o = align_up(o + (vcounts ? NB * 4 : 0), 16);  // counts at vmax (low 16 bits) / vmin (high 16 bits)
    L.off_spec = o;   o = align_up(o + SPEC_CAP * 8, 16);
    L.off_spect = o;  o = align_up(o + SPEC_CAP * 4, 16);
    L.off_exp = o;    o = align_up(o + 32 * 8, 16);        // expf's 2^(i/32) table
    L.off_misc = o;   o = align_up(o + (int)sizeof(Misc), 16);
    L.total = o;
    return L;
}

}  // namespace qs

#endif
