/* qsamp_oracle.c -- TEST INFRASTRUCTURE ONLY (checker, never the product).
 *
 * Plain-C restatement of rye-001/Qwenium's per-step token selection
 * (src/sampling/sampling.cpp), evaluated the way its source reads: every
 * float operation separately rounded, sums accumulated sequentially in
 * sorted order (compiled with -ffp-contract=off, no -ffast-math). It is
 * pinned against the reference itself (oracle/_ref/libqwref_strict.so, the
 * unmodified sources at -O2) by tests/test_oracle_vs_reference.py.
 *
 * Stage order per row (reference file:line in brackets):
 *   soft-cap (extension; a ggml graph op in the reference:
 *             layers/attention.cpp:30-36, models/gemma2.cpp:228-229)
 *   stuck-grammar EOS forcing           [sampling.cpp:40-60]
 *   allow-mask (pruning + grammar)      [sampling.cpp:12-18, 62-80]
 *   repetition penalty                  [sampling.cpp:124-135 / 85-96]
 *   frequency / presence (extension; no reference code)
 *   T <= 0 -> first argmax              [sampling.cpp:149-152 / 106-107]
 *   logits /= T                         [sampling.cpp:154-156]
 *   sort desc, top-k                    [sampling.cpp:158-166]
 *   top-p, float sequential sums        [sampling.cpp:168-179]
 *   softmax over survivors              [sampling.cpp:181-190]
 *   std::discrete_distribution draw     [sampling.cpp:192-193]
 *
 * Choices where the reference is silent or undefined:
 *   - std::sort is unstable; equal logits are ordered here by ascending id.
 *     Tests compare the reference modulo permutations inside a tie group.
 *   - the draw restates libstdc++'s discrete_distribution (GCC 13.3,
 *     <bits/random.tcc>): weights widened to double, divided by their
 *     sequential double sum, partial sums, last entry forced to 1.0,
 *     lower_bound(u); fewer than two weights -> index 0 without drawing.
 *   - soft-cap's tanh is the correctly rounded float tanh ((float)tanhl).
 *   - a row whose every logit is -inf returns the first sorted id (id 0 for
 *     greedy, as max_element does); the reference's weights are NaN there.
 *   - NaN logits are outside the contract (the reference's comparisons are
 *     undefined on them).
 */
#include "qsamp_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

float qso_expf(float x) { return expf(x); }

float qso_bf16_to_f32(uint16_t b) {
    uint32_t w = (uint32_t)b << 16;
    float f;
    memcpy(&f, &w, 4);
    return f;
}

/* ggml's build_softcap: scale by (1/cap), tanh, scale by cap, each in float. */
float qso_softcap(float x, float cap) {
    const float inv = 1.0f / cap;
    const float y = x * inv;
    const float th = (float)tanhl((long double)y);
    return cap * th;
}

typedef struct {
    float l;
    int32_t id;
} entry;

/* descending value, then ascending id; -inf sorts last. */
static int cmp_entry(const void* a, const void* b) {
    const entry* x = (const entry*)a;
    const entry* y = (const entry*)b;
    if (x->l > y->l) return -1;
    if (x->l < y->l) return 1;
    return (x->id > y->id) - (x->id < y->id);
}

static int cmp_i32(const void* a, const void* b) {
    const int32_t x = *(const int32_t*)a, y = *(const int32_t*)b;
    return (x > y) - (x < y);
}

/* The last min(lookback, len) ids; a negative lookback behaves like
 * static_cast<size_t>(lookback), i.e. the whole history. */
static int window_start(int32_t lookback, int len) {
    size_t lb = (size_t)(int64_t)lookback;
    size_t n = (size_t)len;
    size_t w = lb < n ? lb : n;
    return len - (int)w;
}

static void transform_row(float* l, const void* logits, int dtype, int V, const qso_row_params* p,
                          const int32_t* hist, int len, const uint32_t* mask, int32_t* scratch) {
    for (int i = 0; i < V; ++i) {
        float x = dtype == 1 ? qso_bf16_to_f32(((const uint16_t*)logits)[i]) : ((const float*)logits)[i];
        if (p->softcap > 0.0f) x = qso_softcap(x, p->softcap);
        l[i] = x;
    }
    if (p->force_token >= 0 && p->force_token < V) {
        for (int i = 0; i < V; ++i) l[i] = -INFINITY;
        l[p->force_token] = 0.0f;
    } else if (mask) {
        for (int i = 0; i < V; ++i)
            if (!((mask[i >> 5] >> (i & 31)) & 1u)) l[i] = -INFINITY;
    }
    if (len <= 0) return;
    const int s = window_start(p->repetition_lookback, len);
    const int n = len - s;
    if (n <= 0) return;
    memcpy(scratch, hist + s, sizeof(int32_t) * (size_t)n);
    qsort(scratch, (size_t)n, sizeof(int32_t), cmp_i32);
    const int rep_on = p->repetition_penalty != 1.0f;
    const int fp_on = p->frequency_penalty != 0.0f || p->presence_penalty != 0.0f;
    for (int a = 0; a < n;) {
        int b = a + 1;
        while (b < n && scratch[b] == scratch[a]) ++b;
        const int32_t id = scratch[a];
        const int cnt = b - a;
        a = b;
        if (id < 0 || id >= V) continue;
        float v = l[id];
        if (rep_on) v = v < 0 ? v * p->repetition_penalty : v / p->repetition_penalty;
        if (fp_on) {
            v = v - (float)cnt * p->frequency_penalty;
            v = v - p->presence_penalty;
        }
        l[id] = v;
    }
}

static void sample_row(const float* l, int V, const qso_row_params* p, double u, qso_result* r,
                       entry* e, float* probs, double* cp, int32_t* top_ids, float* top_probs,
                       int top_cap) {
    memset(r, 0, sizeof(*r));
    if (p->temperature <= 0.0f) {
        int best = 0;
        for (int i = 1; i < V; ++i)
            if (l[best] < l[i]) best = i;
        r->token = best;
        r->position = 0;
        r->n_keep = 1;
        r->max_logit = l[best];
        r->prob = 1.0f;
        if (top_ids && top_cap > 0) {
            top_ids[0] = best;
            top_probs[0] = 1.0f;
        }
        return;
    }
    for (int i = 0; i < V; ++i) {
        e[i].l = l[i];
        e[i].id = i;
    }
    qsort(e, (size_t)V, sizeof(entry), cmp_entry);
    int n = V;
    if (p->top_k > 0 && p->top_k < V) n = p->top_k;
    const float max_l = e[0].l;
    r->max_logit = max_l;
    if (max_l == -INFINITY) {
        r->token = e[0].id;
        r->n_keep = n;
        r->prob = NAN;
        return;
    }
    if (p->top_p > 0.0f && p->top_p < 1.0f) {
        float sum_exp = 0.0f;
        for (int i = 0; i < n; ++i) sum_exp += qso_expf(e[i].l - max_l);
        float cum = 0.0f;
        int cutoff = n;
        for (int i = 0; i < n; ++i) {
            cum += qso_expf(e[i].l - max_l) / sum_exp;
            if (cum >= p->top_p) {
                cutoff = i + 1;
                break;
            }
        }
        r->sum_exp = sum_exp;
        n = cutoff;
    }
    float sum_keep = 0.0f;
    for (int i = 0; i < n; ++i) {
        const float x = qso_expf(e[i].l - max_l);
        probs[i] = x;
        sum_keep += x;
    }
    for (int i = 0; i < n; ++i) probs[i] /= sum_keep;
    r->sum_keep = sum_keep;
    r->n_keep = n;
    int j = 0;
    if (n >= 2) {
        double dsum = 0.0;
        for (int i = 0; i < n; ++i) dsum += (double)probs[i];
        double acc = 0.0;
        for (int i = 0; i < n; ++i) {
            acc += (double)probs[i] / dsum;
            cp[i] = acc;
        }
        cp[n - 1] = 1.0;
        int lo = 0, hi = n; /* first cp[j] >= u */
        while (lo < hi) {
            const int mid = lo + (hi - lo) / 2;
            if (cp[mid] < u) lo = mid + 1;
            else hi = mid;
        }
        j = lo;
        r->drew = 1;
    }
    r->position = j;
    r->token = e[j].id;
    r->prob = probs[j];
    if (top_ids) {
        const int m = n < top_cap ? n : top_cap;
        for (int i = 0; i < m; ++i) {
            top_ids[i] = e[i].id;
            top_probs[i] = probs[i];
        }
    }
}

typedef struct {
    const void* logits;
    int dtype, B, V;
    int64_t row_stride;
    const qso_row_params* params;
    const int32_t* hist;
    int hist_stride;
    const int32_t* hist_len;
    const uint32_t* masks;
    int64_t mask_stride;
    const double* u;
    qso_result* out;
    int32_t* top_ids;
    float* top_probs;
    int top_cap;
    float* logits_out;
    int next; /* next row to claim (atomic) */
    int fail;
} batch_job;

static void* batch_worker(void* arg) {
    batch_job* j = (batch_job*)arg;
    const int V = j->V;
    const size_t esz = j->dtype == 1 ? 2 : 4;
    float* l = (float*)malloc(sizeof(float) * (size_t)V);
    entry* e = (entry*)malloc(sizeof(entry) * (size_t)V);
    float* probs = (float*)malloc(sizeof(float) * (size_t)V);
    double* cp = (double*)malloc(sizeof(double) * (size_t)V);
    int32_t* scratch = (int32_t*)malloc(sizeof(int32_t) * (size_t)(j->hist_stride > 0 ? j->hist_stride : 1));
    if (!l || !e || !probs || !cp || !scratch) {
        __atomic_store_n(&j->fail, 1, __ATOMIC_RELAXED);
    } else {
        for (int b = __atomic_fetch_add(&j->next, 1, __ATOMIC_RELAXED); b < j->B;
             b = __atomic_fetch_add(&j->next, 1, __ATOMIC_RELAXED)) {
            const void* row = (const char*)j->logits + (size_t)b * (size_t)j->row_stride * esz;
            const int len = j->hist && j->hist_len ? j->hist_len[b] : 0;
            const int32_t* h = j->hist ? j->hist + (size_t)b * (size_t)j->hist_stride : NULL;
            const uint32_t* m = j->masks ? j->masks + (size_t)b * (size_t)j->mask_stride : NULL;
            const qso_row_params* p = &j->params[b];
            transform_row(l, row, j->dtype, V, p, h, len, m, scratch);
            const float T = p->temperature;
            if (T > 0.0f)
                for (int i = 0; i < V; ++i) l[i] /= T;
            if (j->logits_out) memcpy(j->logits_out + (size_t)b * (size_t)V, l, sizeof(float) * (size_t)V);
            sample_row(l, V, p, j->u ? j->u[b] : 0.0, &j->out[b], e, probs, cp,
                       j->top_ids ? j->top_ids + (size_t)b * (size_t)j->top_cap : NULL,
                       j->top_probs ? j->top_probs + (size_t)b * (size_t)j->top_cap : NULL, j->top_cap);
        }
    }
    free(l);
    free(e);
    free(probs);
    free(cp);
    free(scratch);
    return NULL;
}

int qso_sample_batch(const void* logits, int dtype, int B, int V, int64_t row_stride,
                     const qso_row_params* params, const int32_t* hist, int hist_stride,
                     const int32_t* hist_len, const uint32_t* masks, int64_t mask_stride,
                     const double* u, qso_result* out, int32_t* top_ids, float* top_probs,
                     int top_cap, float* logits_out, int n_threads) {
    if (!logits || !params || !out || B < 0 || V <= 0 || row_stride < V) return -1;
    if (dtype != 0 && dtype != 1) return -2;
    batch_job job = {logits, dtype, B, V, row_stride, params, hist, hist_stride, hist_len, masks,
                     mask_stride, u, out, top_ids, top_probs, top_cap, logits_out, 0, 0};
    if (n_threads < 1) n_threads = 1;
    if (n_threads > B) n_threads = B > 0 ? B : 1;
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)n_threads);
    if (!th) return -3;
    int started = 0; /* threads th[0..started) are running */
    for (int t = 1; t < n_threads; ++t) {
        if (pthread_create(&th[started], NULL, batch_worker, &job) != 0) break;
        ++started;
    }
    batch_worker(&job);
    for (int t = 0; t < started; ++t) pthread_join(th[t], NULL);
    free(th);
    return job.fail ? -3 : 0;
}
