/* qsamp_oracle.h -- TEST INFRASTRUCTURE ONLY: CPU restatement of the
 * reference's per-step token selection, used by tests/, smoke() and
 * bench.py's cpu_baseline leg as the checker. The product never links it.
 *
 * The row-parameter struct mirrors the layout of qsamp_row_params in
 * include/qsamp.h so one numpy record array feeds both; it is declared here
 * independently so that the oracle does not depend on product headers.
 */
#ifndef QSAMP_ORACLE_H
#define QSAMP_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    float temperature;          /* <= 0: greedy (argmax after penalties)   */
    int32_t top_k;              /* 0 (or >= V): off                         */
    float top_p;                /* active when 0 < p < 1                    */
    float repetition_penalty;   /* 1.0: off                                 */
    int32_t repetition_lookback;/* window = last min(lookback, len) ids     */
    float frequency_penalty;    /* extension: l -= count * f                */
    float presence_penalty;     /* extension: l -= p if count > 0           */
    float softcap;              /* extension: cap * tanh(l / cap); 0: off   */
    int32_t force_token;        /* >= 0: grammar stuck, only this id (= 0)  */
    int32_t flags;              /* reserved, 0                              */
    uint64_t seed;              /* device RNG mode only; unused here        */
} qso_row_params;

typedef struct {
    int32_t token;      /* selected vocabulary id                               */
    int32_t position;   /* rank of token in the sorted survivor list            */
    int32_t n_keep;     /* survivors after top-k / top-p (1 when greedy)        */
    int32_t drew;       /* 1 if the discrete draw consumed u                    */
    float sum_exp;      /* top-p denominator (sampling.cpp:171); 0 if unused    */
    float sum_keep;     /* softmax denominator over survivors (sampling.cpp:184)*/
    float max_logit;    /* sorted[0] after temperature                          */
    float prob;         /* probability of the selected token                    */
} qso_result;

/* logits: dtype 0 = float32, 1 = bfloat16 (raw uint16 bits); rows of V with
 * row_stride elements. hist: [B][hist_stride] ids, hist_len[B] valid (the
 * newest id last). masks: NULL, or packed uint32 allow-bits, bit i%32 of word
 * i/32, mask_stride words per row (0: one mask shared by all rows). u: [B]
 * uniform draws (the reference engine's generate_canonical value).
 * top_ids/top_probs: optional [B][top_cap] sorted survivor prefix.
 * logits_out: optional [B][V] logits after the transform stage (the values
 * the reference sorts). Returns 0, or a negative code on bad arguments. */
int qso_sample_batch(const void* logits, int dtype, int B, int V, int64_t row_stride,
                     const qso_row_params* params, const int32_t* hist, int hist_stride,
                     const int32_t* hist_len, const uint32_t* masks, int64_t mask_stride,
                     const double* u, qso_result* out, int32_t* top_ids, float* top_probs,
                     int top_cap, float* logits_out, int n_threads);

/* The scalar building blocks, exported so tests can pin them one by one. */
float qso_expf(float x);                 /* glibc expf, as the reference calls it */
float qso_softcap(float x, float cap);   /* cap * tanh_cr(x * (1/cap))            */
float qso_bf16_to_f32(uint16_t b);

#ifdef __cplusplus
}
#endif
#endif
