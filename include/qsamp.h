/* qsamp.h -- C ABI of the B200 token-selection library (libqsamp.so).
 *
 * Replaces the per-step token selection of rye-001/Qwenium
 * (src/sampling/sampling.{h,cpp}) with a batched sm_100a kernel pipeline.
 * Plain C types only; every entry point returns a qsamp_status and never
 * throws. Reference citations are path:line in the Qwenium tree.
 *
 * Semantics per row (the reference's stage order, sampling.cpp:137-194):
 *   soft-cap (Gemma-2 style cap*tanh(x/cap), a model-graph op in the
 *   reference, layers/attention.cpp:30-36) -> allow-mask (vocab pruning
 *   sampling.cpp:12-18, grammar sampling.cpp:25-81) -> repetition penalty
 *   (sampling.cpp:124-135) -> frequency/presence penalty (extension) ->
 *   T <= 0: first argmax | x /= T -> sort -> top-k -> top-p -> softmax ->
 *   discrete draw against u (sampling.cpp:158-193).
 * Results are bit-identical to the reference evaluated in source order
 * (IEEE float, sequential sums); equal logits are ordered by ascending id.
 */
#ifndef QSAMP_H
#define QSAMP_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    QSAMP_OK = 0,
    QSAMP_ERR_INVALID_ARG = 1, /* message names the argument, expected and actual values */
    QSAMP_ERR_CUDA = 2,        /* a CUDA runtime call failed */
    QSAMP_ERR_UNSUPPORTED = 3, /* valid request this build does not serve (message says which) */
    QSAMP_ERR_DEVICE = 4,      /* the kernel reported an internal limit (message says which) */
    QSAMP_ERR_NO_MEMORY = 5,
    QSAMP_ERR_IO = 6,          /* keep-list file unreadable (vocab_utils.h:12-37 throws) */
    QSAMP_ERR_TIMEOUT = 7,     /* a collective did not complete by its deadline (qsamp_comm.h) */
    QSAMP_ERR_COMM = 8         /* a collective failed or its communicator was aborted (qsamp_comm.h) */
} qsamp_status;

typedef enum { QSAMP_F32 = 0, QSAMP_BF16 = 1 } qsamp_dtype;

/* Per-row sampling parameters: one TemperatureSampler / GreedySampler
 * configuration (sampling.h:53-93) per slot. 48 bytes, naturally aligned. */
typedef struct qsamp_row_params {
    float temperature;           /* <= 0: greedy (sampling.cpp:149-152)               */
    int32_t top_k;               /* 0 or >= V: off (sampling.cpp:165-166)             */
    float top_p;                 /* active when 0 < p < 1 (sampling.cpp:168-179)      */
    float repetition_penalty;    /* 1.0: off (sampling.cpp:124-135)                   */
    int32_t repetition_lookback; /* window = last min(lookback, len) ids               */
    float frequency_penalty;     /* extension: l -= count(id) * f over the window      */
    float presence_penalty;      /* extension: l -= p for ids present in the window    */
    float softcap;               /* extension: cap * tanh(l / cap) first; 0: off       */
    int32_t force_token;         /* >= 0: stuck grammar, only this id (logit 0.0),
                                    sampling.cpp:40-60; -1: off                        */
    int32_t flags;               /* reserved, must be 0                                */
    uint64_t seed;               /* Philox key when the batch has no u                 */
} qsamp_row_params;

/* Per-row outcome (device memory). */
typedef struct qsamp_row_result {
    int32_t token;    /* selected id (Sampler::sample's return value)                 */
    int32_t position; /* rank of token among the sorted survivors                     */
    int32_t n_keep;   /* survivors after top-k/top-p (1 when greedy)                  */
    int32_t drew;     /* 1 if the discrete draw consumed u (2+ survivors)             */
    float sum_exp;    /* top-p denominator (sampling.cpp:171); 0 when top-p is off    */
    float sum_keep;   /* softmax denominator over survivors (sampling.cpp:184)        */
    float max_logit;  /* largest logit after temperature                              */
    float prob;       /* probability of token                                         */
} qsamp_row_result;

typedef struct qsamp_ctx qsamp_ctx;

/* One batched selection step: the body of the server's batched decode loop
 * (http_server.cpp:300-306 calls Sampler::sample once per slot; this call
 * serves all slots of a BatchedDecodeFunc step, inference_server.h:177-178). */
typedef struct qsamp_batch {
    const void* logits;               /* DEVICE [B][row_stride] of dtype (the output
                                         head's [V,B] tensor, forward_pass_base.cpp:138-158) */
    qsamp_dtype dtype;
    int32_t B, V;
    int64_t row_stride;               /* elements between rows, >= V                  */
    const qsamp_row_params* params;   /* HOST [B]                                     */
    const int32_t* hist;              /* DEVICE [B][hist_stride] ids, newest last, or NULL */
    int32_t hist_stride;
    const int32_t* hist_len;          /* HOST [B] valid ids per row (NULL: hist_stride) */
    const uint32_t* masks;            /* DEVICE allow-bits, bit i%32 of word i/32, or NULL */
    int64_t mask_stride;              /* words between row masks; 0: one shared mask   */
    const double* u;                  /* HOST [B] uniforms in [0,1), or NULL: Philox    */
    uint64_t rng_offset;              /* Philox counter offset (when u is NULL)         */
    int32_t* out_ids;                 /* DEVICE [B] or NULL                             */
    qsamp_row_result* out_results;    /* DEVICE [B] or NULL                             */
    int32_t* out_top_ids;             /* DEVICE [B][top_cap] sorted survivors, or NULL  */
    float* out_top_probs;             /* DEVICE [B][top_cap], or NULL                   */
    int32_t top_cap;
} qsamp_batch;

/* Context bound to one CUDA device (ownership as in sampling.h:46-50: the
 * sampler owns its scratch; all batch pointers are borrowed for the call). */
qsamp_status qsamp_create(int32_t device, qsamp_ctx** out);
void qsamp_destroy(qsamp_ctx* ctx);
/* Last error message of this context (valid until the next call). */
const char* qsamp_last_error(const qsamp_ctx* ctx);

/* Batched selection, stream-ordered on `stream` (a cudaStream_t; NULL: the
 * legacy default stream). Replaces the per-slot loop of
 * QwenServerIntegration::run_batched_decode (http_server.cpp:300-306). */
qsamp_status qsamp_sample(qsamp_ctx* ctx, const qsamp_batch* batch, void* stream);

/* The same with every pointer in HOST memory (logits, hist, masks, outputs):
 * copies in, selects, copies out, synchronises. This is the drop-in for
 * Sampler::sample(std::vector<float>& logits, ...) (sampling.h:22-24), whose
 * logits live on the host. */
qsamp_status qsamp_sample_host(qsamp_ctx* ctx, const qsamp_batch* batch);

/* Device-side outcome of the most recent qsamp_sample, qsamp_shard_topk or
 * qsamp_merge_topk call on this context. Those calls are asynchronous and
 * return before the kernels run; each ends with a stream-ordered copy of the
 * kernels' status word into pinned host memory, which this function reads.
 * Call it after synchronising that call's stream. QSAMP_OK, or
 * QSAMP_ERR_DEVICE with qsamp_last_error naming the limit that was hit (a
 * gather-round budget, a bounded wait that ran out); the rows concerned
 * carry token -1. The reference throws where a row cannot be sampled
 * (sampling.cpp:101,140): a caller that replaces Sampler::sample with
 * qsamp_sample converts QSAMP_ERR_DEVICE into that throw.
 * (qsamp_sample_host reads the status itself and returns it.) */
qsamp_status qsamp_poll_status(qsamp_ctx* ctx);

/* Device-side limits of a context (no counterpart in the reference). The
 * kernels never wait without a bound; these set the bounds:
 *   max_rounds      gather rounds a full-vocabulary row may take before it
 *                   is given up (token -1, QSAMP_ERR_DEVICE); default 64,
 *                   at least 1.
 *   ready_wait_ns   qsamp_sample_host copies the logits in row chunks while
 *                   the kernels run; a kernel waits at most this long for a
 *                   chunk's arrival flag before it gives the row up
 *                   (token -1); default 1e9 (one second), at least 1000.
 *   drop_ready_from fault injection for tests: chunks with index >= this
 *                   value never raise their arrival flag (their bytes are
 *                   still copied), so the kernels' bounded waits run out;
 *                   -1 (the default) turns it off.
 *   hist_path       1 (the default): bf16 rows with a full-vocabulary top-p
 *                   take the histogram kernel; 0: the cluster kernel serves
 *                   them (both give the same rows bit for bit).
 *   live_path       0 (the default): the cluster kernel serves fp32 rows with
 *                   a full-vocabulary top-p; 1: they are shared between the
 *                   cluster kernel and the live-list kernel, which serves a
 *                   row whose elements within 17.5 of its maximum number at
 *                   most 4096 on one SM (qsamp_sample only; the host entry
 *                   point keeps them on the cluster kernel). Worth turning on
 *                   for peaked rows (low temperatures, confident models):
 *                   measured on B200 with the config2 batches at temperatures
 *                   0.2-0.6, 9% less time per call; at 0.2-1.2, 1-3% more.
 *                   2 (tests): the live-list kernel returns every row it
 *                   takes, and a second cluster launch serves them. All give
 *                   the same rows bit for bit. */
typedef struct qsamp_limits {
    int32_t max_rounds;
    int32_t drop_ready_from;
    int64_t ready_wait_ns;
    int32_t hist_path;
    int32_t live_path;
} qsamp_limits;
qsamp_status qsamp_set_limits(qsamp_ctx* ctx, const qsamp_limits* limits);
qsamp_status qsamp_get_limits(const qsamp_ctx* ctx, qsamp_limits* out);

/* Allocation-free selection. No counterpart in the reference: it exists
 * for callers that may not allocate device memory when they sample (a
 * serving engine that reserves all device memory up front for its own
 * allocator, a plugin host that forbids cudaMalloc). qsamp_create
 * allocates, so this entry point takes no context.
 *
 * Same batch semantics as qsamp_sample (logits, hist, masks and outputs in
 * device memory; params, hist_len and u on the host). Its scratch is one
 * static device array of QSAMP_STATIC_SCRATCH_BYTES that every GPU loading
 * the library holds until the process exits; it serves at most
 * QSAMP_STATIC_MAX_ROWS rows per call (more: QSAMP_ERR_INVALID_ARG) and one
 * bf16 soft-cap table per call (rows with a second cap value compute tanh per
 * logit). The first call on a device, with that device current, looks up the
 * array's device address; make it before any stream capture. All calls on a
 * device share the array, so calls whose work overlaps on the GPU race.
 * Device-side limits (the gather-round budget of a full-vocabulary row, a
 * slice copy that did not complete) are reported only in the row results:
 * token -1 for that row; the call has no other channel for them. err, when
 * non-NULL, receives a message of at most err_len bytes. */
#define QSAMP_STATIC_MAX_ROWS 4096
#define QSAMP_STATIC_SCRATCH_BYTES (640u * 1024u)
qsamp_status qsamp_sample_static(const qsamp_batch* batch, void* stream, char* err, size_t err_len);

/* Host helpers for the allow-mask. -------------------------------------- */

/* Pack ids into allow-bits (words = ceil(V/32), zeroed first); ids outside
 * [0,V) are ignored. Replaces the vector<bool> of sampling.cpp:62-64 and the
 * keep-set lookup of apply_vocab_pruning (sampling.cpp:12-18). */
qsamp_status qsamp_pack_ids(const int32_t* ids, int64_t n, int32_t V, uint32_t* mask_out);

/* The grammar allow-mask of Sampler::apply_grammar_constraints
 * (sampling.cpp:25-81) from GrammarVocab::get_valid_tokens ids
 * (grammar_vocab.cpp:571-755): valid ids; if `accepting`, also
 * eos_string_id (the first vocab entry equal to "<|endoftext|>" or
 * "<|im_end|>", see qsamp_find_eos_string) and eos_token_id when in range.
 * With no valid id the grammar is stuck: *force_token_out = eos_string_id
 * (logit forced to 0.0, all others -inf) and the mask is cleared; otherwise
 * *force_token_out = -1. */
qsamp_status qsamp_grammar_mask(const int32_t* valid_ids, int64_t n_valid, int32_t accepting,
                                int32_t eos_string_id, int32_t eos_token_id, int32_t V,
                                uint32_t* mask_out, int32_t* force_token_out);

/* First id whose string is "<|endoftext|>" or "<|im_end|>" (the scan of
 * sampling.cpp:53-58 and :67-71), or -1. strs[i] has lens[i] bytes. */
int32_t qsamp_find_eos_string(const char* const* strs, const int32_t* lens, int32_t V);

/* Vocab-pruning keep list, file format [u32 count][u32 id]*count
 * (load_keep_list, vocab_utils.h:12-37), packed into allow-bits. */
qsamp_status qsamp_keep_list_mask(const char* path, int32_t V, uint32_t* mask_out);

/* AND two allow-masks word by word (pruning AND grammar). */
qsamp_status qsamp_mask_and(const uint32_t* a, const uint32_t* b, int64_t words, uint32_t* out);

/* Grammar char classes on the device. ------------------------------------
 * TokenTrie::mark_char_class (token-trie.cpp:93-116) marks every token whose
 * FIRST byte the class allows (empty tokens are never marked, token-trie.cpp
 * :18); GrammarVocab::get_valid_tokens calls it once per distinct char class
 * among the grammar's stacks (grammar_vocab.cpp:589-597), ~150K ids for a
 * negated class such as [^"]. Here the marks of B grammar states are made at
 * once on the GPU, straight into the allow-masks qsamp_sample reads.
 *
 * qsamp_first_byte_table (host): table[i] = first byte of token i (0..255),
 * 256 for an empty token; copy it to the device once per vocabulary.
 * qsamp_char_class_masks: for row b, bit i of masks[b] is set when token i's
 * first byte is allowed by classes[b] (256 bits, bit c%32 of word c/32, with a
 * negated class already complemented); or_into = 1 ORs into the existing
 * words (a state with several char classes, or literal ids packed before),
 * 0 overwrites them. table, classes [B][8] and masks [B][mask_stride] are
 * DEVICE pointers; stream-ordered. No counterpart of the batching in the
 * reference (its marks are per state, on the host). */
qsamp_status qsamp_first_byte_table(const char* const* strs, const int32_t* lens, int32_t V, uint16_t* table_out);
qsamp_status qsamp_char_class_masks(qsamp_ctx* ctx, const uint16_t* table, int32_t V, int32_t B,
                                    const uint32_t* classes, uint32_t* masks, int64_t mask_stride, int32_t or_into,
                                    void* stream);

/* Compact token trie (host). ----------------------------------------------
 * The queries of the reference's qwenium::TokenTrie (token-trie.h:20-64,
 * token-trie.cpp:8-126) with identical results in identical order, over a
 * flat sorted-string representation instead of 256-pointer nodes
 * (token-trie.h:11-16). C++ callers use qwenium_b200/trie/token-trie.h,
 * a drop-in qwenium::TokenTrie; this is the C ABI over the same code.
 * qsamp_trie_build: token i is strs[i] (lens[i] bytes); empty tokens are
 * skipped (token-trie.cpp:18). The collect functions write at most cap ids
 * into out and return how many the query yields (-1: invalid argument):
 *   by_prefix     collect_by_prefix(prefix[0:len], offset)  (token-trie.cpp:39-70)
 *   by_char_class collect_by_char_class(set of chars[0:n], negated)  (:72-84)
 *   by_first_char collect_by_first_char(c)  (:86-91)
 * qsamp_trie_mark_char_class sets mask_out[i] = 1 for the marked tokens and
 * 0 elsewhere (mark_char_class, :93-116); V must cover every marked id. */
typedef struct qsamp_trie qsamp_trie;
qsamp_status qsamp_trie_build(const char* const* strs, const int32_t* lens, int32_t V, qsamp_trie** out);
void qsamp_trie_free(qsamp_trie* trie);
int64_t qsamp_trie_token_count(const qsamp_trie* trie);
int64_t qsamp_trie_memory_bytes(const qsamp_trie* trie);
int64_t qsamp_trie_collect_by_prefix(const qsamp_trie* trie, const char* prefix, int32_t len, int32_t offset,
                                     int32_t* out, int64_t cap);
int64_t qsamp_trie_collect_by_char_class(const qsamp_trie* trie, const uint8_t* chars, int32_t n, int32_t negated,
                                         int32_t* out, int64_t cap);
int64_t qsamp_trie_collect_by_first_char(const qsamp_trie* trie, uint8_t c, int32_t* out, int64_t cap);
qsamp_status qsamp_trie_mark_char_class(const qsamp_trie* trie, const uint8_t* chars, int32_t n, int32_t negated,
                                        int32_t V, uint8_t* mask_out);

/* Vocab-sharded selection (tensor-parallel output head). No counterpart in
 * the reference (its sampler sees whole rows). ----------------------------
 * Rank r holds logits[:, v_offset : v_offset + V_local] of a V_total vocab
 * (local_batch->V = V_local, row_stride in local elements).
 * Step 1, qsamp_shard_topk on each rank: the row transform (soft-cap, allow
 * mask, penalties, /T) and the local top-k as (value, global id) pairs sorted
 * by (value desc, id asc) into DEVICE cand_vals / cand_ids [B][k], padded with
 * (-inf, -1). hist and force_token hold GLOBAL ids; masks cover the local
 * slice (bit i <-> global id v_offset + i). Every temperature row needs
 * 0 < top_k <= k and top_k < V_total (a full-vocabulary top-p is served by
 * the unsharded path only: QSAMP_ERR_UNSUPPORTED); penalty windows <= 1024;
 * 1 <= k <= 1024. u and the batch's outputs are not used.
 * Step 2: an all-gather of the [B][k] blocks over the ranks (NCCL), giving
 * DEVICE all_vals / all_ids [n_ranks][B][k] rank-major, then
 * qsamp_merge_topk on every rank: the global top-k of the union (ties to the
 * lower global id), top-p, softmax and the draw. With top_k > 0 the
 * reference's top-p and softmax see only the top-k set (sampling.cpp:158-190),
 * so the rows equal the unsharded path's bit for bit. params and u are HOST
 * [B]; n_ranks * k <= 5120. Slices must not overlap. */
qsamp_status qsamp_shard_topk(qsamp_ctx* ctx, const qsamp_batch* local_batch, int32_t v_offset,
                              int32_t V_total, int32_t k, float* cand_vals, int32_t* cand_ids,
                              void* stream);
qsamp_status qsamp_merge_topk(qsamp_ctx* ctx, int32_t n_ranks, int32_t B, int32_t k,
                              const float* all_vals, const int32_t* all_ids,
                              const qsamp_row_params* params, const double* u, uint64_t rng_offset,
                              int32_t* out_ids, qsamp_row_result* out_results, void* stream);

/* Greedy verification of prompt-lookup drafts (speculative decoding). -----
 * SpeculativeDecoder::try_speculative_step (speculative.h:150-239) runs a
 * slot's K draft tokens through the model in one pass and accepts them
 * greedily: row i of the K logits rows must predict draft[i+1]
 * (argmax, speculative.h:248-258: the first maximum, NaN never larger, a NaN
 * at index 0 wins), an accepted EOS draft stops the step, and the bonus token
 * is the argmax at the first mismatch or after the last row. Here the rows of
 * B slots are verified at once on the device. Slot b owns rows
 * [row_off[b], row_off[b+1]) of logits (DEVICE [n_rows][row_stride], dtype)
 * and the same entries of drafts; row_off (DEVICE [B+1], row_off[0] = 0,
 * row_off[B] = n_rows). Outputs (DEVICE [B]): accepted (draft tokens kept),
 * bonus (or -1), has_bonus (bonus != eos_token). K = 0: 0, -1, 0 (no draft).
 * No counterpart of the batching in the reference (one slot per call). */
qsamp_status qsamp_verify_greedy(qsamp_ctx* ctx, const void* logits, qsamp_dtype dtype, int32_t V, int64_t row_stride,
                                 int32_t n_rows, int32_t B, const int32_t* row_off, const int32_t* drafts,
                                 int32_t eos_token, int32_t* out_accepted, int32_t* out_bonus,
                                 int32_t* out_has_bonus, void* stream);

/* Counters since creation (observability). No counterpart in the
 * reference. kernel_launches counts every kernel this context launched
 * (selection, merge, soft-cap tables). With kernel timing on, each selection
 * kernel launch is bracketed by CUDA events on the call's stream and
 * qsamp_get_counters waits for the last call's events and reports their
 * device times (0 for a kernel the call did not launch); timing off (the
 * default) records nothing and qsamp_get_counters never waits. */
typedef struct qsamp_counters {
    uint64_t calls, rows, logit_bytes, gather_rounds;
    double last_call_us;
    uint64_t kernel_launches;
    double last_stream_kernel_ms; /* greedy / top-k rows, and vocab shards */
    double last_rows_kernel_ms;   /* full-vocabulary rows (cluster kernel) */
    double last_merge_kernel_ms;  /* qsamp_merge_topk */
    /* routing and launch shape of the last qsamp_sample / qsamp_sample_host
     * call: rows served by the stream kernel and by the cluster kernel, the
     * cluster kernel's CTAs per cluster and clusters launched (0 when it did
     * not run) */
    int32_t last_stream_rows, last_cluster_rows;
    int32_t last_cluster_size, last_clusters;
    /* bf16 full-vocabulary rows given to the histogram kernel, how many of
     * them it handed on to the cluster kernel (read from the last call's
     * stream-ordered status copy: valid once that call's stream is
     * synchronised), and its device time */
    int32_t last_hist_rows, last_hist_handed_on;
    double last_hist_kernel_ms;
    /* fp32 full-vocabulary rows offered to the live-list kernel, how many it
     * served and how many it returned to the cluster kernel (stream-ordered
     * copies, valid once the call's stream is synchronised), and its device
     * time */
    int32_t last_live_candidates, last_live_rows, last_live_returned, reserved0;
    double last_live_kernel_ms;
} qsamp_counters;
qsamp_status qsamp_get_counters(const qsamp_ctx* ctx, qsamp_counters* out);
qsamp_status qsamp_set_kernel_timing(qsamp_ctx* ctx, int32_t on);

#ifdef __cplusplus
}
#endif
#endif /* QSAMP_H */
