/*
 * hkv.h -- C ABI of the B200 paged KV-cache decode engine.
 *
 * The engine replaces the per-request KV-slot path of higgs-audio.cpp
 * (src/higgs_pipeline.cpp): the slot arena (BackendKvCache / BackendRuntime,
 * :326-403, :1137-1220), the K/V row write into the cache (ggml_set_inplace,
 * :5748-5749 decode, :6278-6279 window, :6603-6604 prefill), the NEOX RoPE on
 * the BF16 table (:471-506) and the GQA decode attention chain (:5750-5786).
 *
 * Storage model: one page pool per engine (per GPU).  A page holds 16
 * consecutive token positions of one slot for ALL layers (one block in each
 * layer's slab), K and V, all KV heads, in F16.  Each live slot owns a page list; pages are reference
 * counted so slots can share a prefix (fork / published prefixes) and are
 * copied on the first write into a shared page (copy-on-write).
 *
 * Conventions:
 *   * Every function returns an hkv_status; on failure hkv_last_error() holds
 *     a message and no slot or page state has changed.
 *   * `slots` arrays are HOST arrays of slot ids.  Tensor arguments of the
 *     compute calls (q, k, v, out, gather outputs) are DEVICE pointers on the
 *     engine's GPU, 16-byte aligned; compute calls are ordered on `stream` (a
 *     cudaStream_t, 0 for the legacy default stream) and return before the
 *     GPU finishes.
 *   * Decode step protocol (one new token per slot):
 *         for layer in [0, n_layers):
 *             hkv_rope_append(layer, ...)   writes row `used` of each slot
 *             hkv_decode_attn(layer, ...)   attends rows [0, used]
 *         hkv_slot_advance(...)             used += 1
 *     This mirrors the reference's `past = cache.used` for all layers of one
 *     graph followed by `cache.used += 1` (:5642, :5183).
 *   * Row layouts follow ggml order: a K/V row is [n_head_kv][head_dim],
 *     q and the attention output are head-major [n_head][head_dim]; query
 *     head h reads KV head h / (n_head / n_head_kv) (:441-456).
 *   * Slot operations are thread-safe (one mutex per engine).  Compute calls
 *     on one engine share its split-partial buffer: issue them on one stream
 *     (or order the streams) in the order the GPU should run them.
 */
#ifndef HKV_H
#define HKV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HKV_ABI_VERSION 3  /* 2: hkv_pool_stats.kernel_launches; 3: tensor_cores in the q4k args,
                              hkv_backbone_kernel_launches */

typedef enum hkv_status {
    HKV_OK = 0,
    HKV_ERR_INVALID = 1,   /* bad argument or unsupported shape              */
    HKV_ERR_OOM = 2,       /* page pool, reservation or slot table exhausted */
    HKV_ERR_BAD_SLOT = 3,  /* slot id not live (or released twice)           */
    HKV_ERR_RANGE = 4,     /* position / length out of range                 */
    HKV_ERR_CUDA = 5,      /* CUDA runtime error                             */
    HKV_ERR_TIMEOUT = 6,   /* a bounded device-side wait gave up             */
    HKV_ERR_NO_DEVICE = 7, /* compute call on a host-only engine             */
    HKV_ERR_NOT_FOUND = 8, /* unknown prefix key                             */
    HKV_ERR_DEVICE = 9     /* a kernel's bounds check recorded a bad index   */
} hkv_status;

typedef struct hkv_engine hkv_engine;
typedef void *hkv_stream; /* cudaStream_t */

/* Engine shape.  Replaces TextConfig fields the KV path reads
 * (include/higgs_audio.h:86-100: block_count, head_count, head_count_kv,
 * key_length, context_length, rope_freq_base) plus pool sizing. */
typedef struct hkv_config {
    int32_t n_layers;       /* 36                                              */
    int32_t n_head;         /* query heads, 32                                 */
    int32_t n_head_kv;      /* KV heads held by this engine, 8 (or a share)    */
    int32_t head_dim;       /* 128 (the only value the kernels take)           */
    int32_t page_tokens;    /* 16 (the only value the kernels take)            */
    int32_t context_length; /* 32768: RoPE table rows and max positions        */
    float rope_freq_base;   /* 1e6                                             */
    int32_t max_slots;      /* slot-table size                                 */
    int64_t n_pages;        /* pages in the pool                               */
    int32_t device;         /* CUDA ordinal; -1 = host-only bookkeeping engine */
    uint32_t shuffle_seed;  /* nonzero: the free list starts in a seeded random
                               order, so logical pages land on scattered
                               physical pages (tests, benchmarks)              */
} hkv_config;

/* Key of a shareable prompt prefix, e.g. a hash of the reference-code cache
 * key (model, reference wav path, size, mtime: :1545-1551) and the
 * reference-prompt token count. */
typedef struct hkv_prefix_key {
    uint64_t hash;
    int64_t n_tokens;
} hkv_prefix_key;

typedef struct hkv_pool_stats {
    int64_t n_pages;       /* pool size                                       */
    int64_t free_pages;    /* on the free list                                */
    int64_t reserved;      /* free pages promised to live slots               */
    int64_t shared_pages;  /* pages with refcount > 1                         */
    int32_t live_slots;
    int32_t prefixes;
    int64_t page_bytes;    /* bytes of one page (all layers, K and V)         */
    int64_t cow_copies;    /* pages copied on write since creation            */
    int64_t kernel_launches; /* kernels this engine enqueued since creation   */
} hkv_pool_stats;

/* Kernel ids for the CUDA-event profiler. */
typedef enum hkv_kernel_id {
    HKV_KERNEL_APPEND = 0,  /* hkv_append, hkv_rope_append, hkv_rope_append_range */
    HKV_KERNEL_ATTN = 1,    /* hkv_decode_attn                                    */
    HKV_KERNEL_COMBINE = 2, /* reserved: nothing is recorded under this id; the
                               combine launch that follows some attention launches
                               is timed with them (ATTN or STEP)              */
    HKV_KERNEL_GATHER = 3,  /* hkv_gather                                         */
    HKV_KERNEL_STEP = 4,    /* hkv_decode_step (append + attention, one launch)   */
    HKV_KERNEL_GEMV = 5,    /* Q4_K projections (hkv_q4k_*, hkv_backbone_decode)  */
    HKV_KERNEL_EMBED = 6,   /* embedding rows (hkv_backbone_embed_*)              */
    HKV_KERNEL_COUNT = 7
} hkv_kernel_id;

/* ------------------------------------------------------------ engine -- */

/* Qwen3-4B / HiggsAudioV3 backbone shape (docs/spec.md:329-341). */
int hkv_config_default(hkv_config *cfg);

/* Creates the pool (one device allocation, zero-filled), the BF16 RoPE tables
 * (make_bf16_rope_table, :475-487, built on the host and uploaded once as in
 * ensure_backend_kv_rope_tables, :1606-1622) and the split-partial buffer. */
int hkv_engine_create(const hkv_config *cfg, hkv_engine **out);
int hkv_engine_destroy(hkv_engine *eng);
/* The configuration the engine was created with. */
int hkv_engine_config(const hkv_engine *eng, hkv_config *out);

/* Message of the last failed call on this engine ("" if none). */
const char *hkv_last_error(const hkv_engine *eng);
const char *hkv_status_string(int status);
int hkv_abi_version(void);

/* ------------------------------------------------------------- slots -- */

/* Rents a slot.  Replaces acquire_backend_kv_cache_slot (:1191-1208).
 * capacity_hint: positions the request will reach (prompt + steps + 1, as
 *   the reference's capacity, :4820); the pages it needs beyond a shared
 *   prefix are reserved so later appends cannot run out (HKV_ERR_OOM here
 *   instead).  0 reserves nothing.
 * share: if non-NULL and published, the slot starts with that prefix's pages
 *   mapped (used = share->n_tokens, copy-on-write); if not published the slot
 *   starts empty (check hkv_slot_len). */
int hkv_slot_acquire(hkv_engine *eng, int64_t capacity_hint, const hkv_prefix_key *share,
                     int32_t *slot_out);

/* Returns a slot.  Replaces ScopedBackendKvCacheSlot::release (:1210-1220).
 * Drops the slot's page references; a second release is HKV_ERR_BAD_SLOT. */
int hkv_slot_release(hkv_engine *eng, int32_t slot);

/* New slot sharing the first n_tokens positions of src (copy-on-write).
 * No reference counterpart (the reference copies whole caches); it is the
 * primitive behind prefix sharing. */
int hkv_slot_fork(hkv_engine *eng, int32_t src, int64_t n_tokens, int32_t *dst_out);

/* cache.used of the reference (:340). */
int hkv_slot_len(const hkv_engine *eng, int32_t slot, int64_t *used_out);

/* Truncates a slot (rollback, e.g. the reference's window refresh that
 * rewrites rows [start, used), :4837-4842).  used must be <= current. */
int hkv_slot_set_len(hkv_engine *eng, int32_t slot, int64_t used);

/* used += n_tokens for each slot (the caller's `cache.used += 1`, :5183,
 * :4925; prefill sets used = P, :4837).  The rows must have been written. */
int hkv_slot_advance(hkv_engine *eng, int32_t n, const int32_t *slots, int64_t n_tokens);

/* Publishes the first key->n_tokens positions of `slot` under `key`; the
 * prefix holds its own page references until hkv_prefix_drop. */
int hkv_prefix_publish(hkv_engine *eng, const hkv_prefix_key *key, int32_t slot);
int hkv_prefix_drop(hkv_engine *eng, const hkv_prefix_key *key);

/* Physical page ids of a slot (diagnostics and tests). */
int hkv_slot_pages(const hkv_engine *eng, int32_t slot, int32_t *pages_out, int64_t cap,
                   int64_t *n_out);
int hkv_pool_stats_get(const hkv_engine *eng, hkv_pool_stats *out);

/* ----------------------------------------------------------- compute -- */

/* Raw K/V row write at position `used` of each slot, for one layer: the
 * drop-in for ggml_set_inplace(cache.key, k_cur) / (cache.value, v_cur)
 * (:5748-5749) when the caller already applied RoPE.  k, v: device
 * [n][n_head_kv][head_dim] F32, stored as F16 (round to nearest even). */
int hkv_append(hkv_engine *eng, int32_t layer, int32_t n, const int32_t *slots, const float *k,
               const float *v, hkv_stream stream);

/* Fused NEOX RoPE (BF16 table, position `used`, :489-506 / :5735) of the
 * pre-RoPE k, then the row write of roped k and raw v.  Same shapes. */
int hkv_rope_append(hkv_engine *eng, int32_t layer, int32_t n, const int32_t *slots,
                    const float *k_prerope, const float *v, hkv_stream stream);

/* Prefill / window writer: positions [used, used + n_tokens) of one slot,
 * one layer (:6603-6604 prefill at 0, :6278-6279 window at start).
 * k_prerope, v: device [n_tokens][n_head_kv][head_dim] F32.  Call for every
 * layer, then hkv_slot_advance(n_tokens). */
int hkv_rope_append_range(hkv_engine *eng, int32_t layer, int32_t slot, int64_t n_tokens,
                          const float *k_prerope, const float *v, hkv_stream stream);

/* GQA decode attention of one new token per slot over rows [0, used]
 * (used + 1 rows, the last one written by this step's append), for one
 * layer.  Replaces repeat_kv_3d + mul_mat + scale(1/sqrt(head_dim)) +
 * soft_max + mul_mat + permute/cont (:5750-5786).  q_prerope: device
 * [n][n_head][head_dim] F32 before RoPE (RoPE at position `used` is applied
 * inside, :5734).  out: device [n][n_head * head_dim] F32, head-major. */
int hkv_decode_attn(hkv_engine *eng, int32_t layer, int32_t n, const int32_t *slots,
                    const float *q_prerope, float *out, hkv_stream stream);

/* hkv_rope_append followed by hkv_decode_attn for one layer, as ONE kernel
 * launch: the warp that owns a slot's last page for a KV head ropes the new
 * K row, writes K and V to the page and patches the copy it attends from.
 * Same shapes and results (cache bits and outputs) as the two calls. */
int hkv_decode_step(hkv_engine *eng, int32_t layer, int32_t n, const int32_t *slots,
                    const float *q_prerope, const float *k_prerope, const float *v, float *out,
                    hkv_stream stream);

/* Logical view of one slot/layer: rows [pos0, pos0 + n) as
 * [n][n_head_kv][head_dim] F16 bits, the layout of the reference's cache
 * rows (:1137-1142).  Test hook replacing ggml_backend_tensor_get on the
 * cache (:6980-6981).  k_out, v_out: device pointers. */
int hkv_gather(hkv_engine *eng, int32_t slot, int32_t layer, int64_t pos0, int64_t n,
               uint16_t *k_out, uint16_t *v_out, hkv_stream stream);

/* Waits for the engine's stream work, then reports a device-side error
 * (HKV_ERR_DEVICE / HKV_ERR_TIMEOUT) recorded by a kernel since the last
 * call, and clears it. */
int hkv_sync_check(hkv_engine *eng, hkv_stream stream);

/* Host copies of the BF16 RoPE tables, [context_length][head_dim/2] each. */
int hkv_rope_tables(const hkv_engine *eng, float *cos_out, float *sin_out);

/* ------------------------------------------------------ KV-head split -- */

/* One long request split by KV head across `world` GPUs, one process and one
 * engine per GPU, each engine holding n_head_kv = (total KV heads) / world of
 * every layer.  The reference has no multi-GPU path (it runs on CUDA device 0,
 * src/higgs_pipeline.cpp:126); this replaces an all-gather of the per-head
 * attention outputs before o_proj with peer stores from inside the decode
 * kernel: every finished head slice is written into every rank's exchange
 * region over NVLink and each rank's per-layer arrival counter is bumped.
 *
 *   hkv_split_export   allocate this rank's exchange region (zeroed) and
 *                      export its CUDA IPC handle (64 bytes) to handle_out
 *   hkv_split_connect  map every peer's region from the world's handles
 *                      (world x 64 bytes, rank order); all ranks must have
 *                      exported before any rank runs hkv_split_step.  With
 *                      handles == NULL it closes the peer mappings: every
 *                      rank must do so (then meet at a barrier) before any
 *                      rank destroys its engine, which frees its region
 *   hkv_split_step     hkv_decode_step over this rank's KV heads (q, k, v hold
 *                      this rank's heads), the outputs going to all ranks
 *   hkv_split_wait     enqueue a bounded wait until every rank's slices of
 *                      this layer's latest step have arrived here; after it,
 *                      work on `stream` may read the output (a peer that
 *                      never delivers ends the wait with HKV_ERR_TIMEOUT at
 *                      the next hkv_sync_check)
 *   hkv_split_output   this rank's full output of one layer, rows of
 *                      row_floats F32 (one row per batch entry, heads in
 *                      global order); each layer has its own block, so a rank
 *                      running ahead never overwrites what a peer still reads
 * Every rank must pass its entries in the same request order. */
int hkv_split_export(hkv_engine *eng, int32_t world, int32_t rank, void *handle_out);
int hkv_split_connect(hkv_engine *eng, const void *handles);
int hkv_split_step(hkv_engine *eng, int32_t layer, int32_t n, const int32_t *slots,
                   const float *q_prerope, const float *k_prerope, const float *v,
                   hkv_stream stream);
int hkv_split_wait(hkv_engine *eng, int32_t layer, hkv_stream stream);
int hkv_split_output(const hkv_engine *eng, int32_t layer, float **out_dev, int64_t *row_floats);

/* ---------------------------------------------------- no allocation -- */

/* Device memory a caller already owns, in the engine's page layout: one slab
 * per layer, each page of a slab {K, V} x n_head_kv head blocks of 16 rows x
 * 128 F16 dims (4 KiB), block(page, layer, kv, head) =
 * ((layer*n_pages + page)*2 + kv)*n_head_kv + head, and row r keeps its
 * 16-byte chunk c at position c ^ (r & 7).
 * rope_cos / rope_sin: [context_length][64] F32 BF16-rounded tables. */
typedef struct hkv_paged_view {
    void *pool;
    int64_t n_pages;
    int32_t n_layers;
    int32_t n_head_kv;
    const float *rope_cos;
    const float *rope_sin;
    int32_t context_length;
} hkv_paged_view;

/* Decode attention that allocates no GPU memory.  No counterpart in the
 * reference: it exists for callers that may not call cudaMalloc -- code that
 * must live inside another framework's device memory pool (for example the
 * pipeline's ggml backend buffers) or on a path where an allocation could
 * block or fail.  Same computation as hkv_decode_attn, on caller-owned pages:
 *   pos[e]: host, the last row slot e attends (rows [0, pos[e]]), which is
 *     also the RoPE position of its query;
 *   page_off[n+1], pages[]: host, slot e's physical pages are
 *     pages[page_off[e] .. page_off[e+1]);
 *   q_prerope [n][4*n_head_kv][128] F32, out [n][4*n_head_kv*128] F32: device.
 * Working memory (plan, split partials, error word) lives in one static
 * device array of 8 MiB per GPU, held until the process exits; a batch that
 * needs more is rejected with HKV_ERR_RANGE and a message in err_msg (which
 * may be NULL).  The first call on a device looks the array's address up
 * (cudaGetSymbolAddress); make that first call before any stream capture.
 * All calls share the array: calls that overlap on the GPU race.  A kernel
 * that gives up on a bounded wait or meets a bad page id records it in the
 * array's error word and returns; the word keeps its first record until
 * hkv_decode_attn_noalloc_sync_check reads it, so check after the calls whose
 * outputs you use. */
int hkv_decode_attn_noalloc(const hkv_paged_view *view, int32_t layer, int32_t n,
                            const int32_t *pos, const int32_t *page_off, const int32_t *pages,
                            const float *q_prerope, float *out, hkv_stream stream,
                            char *err_msg, size_t err_len);

/* The error check of hkv_decode_attn_noalloc (also no counterpart in the
 * reference, and it allocates nothing either): synchronises `stream`, reads
 * the static array's error word on the current device and clears it.
 * HKV_OK if no call since the last check recorded an error; HKV_ERR_TIMEOUT
 * (a bounded wait gave up) or HKV_ERR_DEVICE (a bad page id reached a kernel)
 * otherwise, with a message in err_msg (which may be NULL): the output of the
 * call that recorded it is invalid. */
int hkv_decode_attn_noalloc_sync_check(hkv_stream stream, char *err_msg, size_t err_len);

/* ------------------------------------------- Q4_K backbone projections -- */
/* The projections around the KV path in the reference's decode graph
 * (src/higgs_pipeline.cpp:5709-5733 q/k/v with per-head RMSNorm, :5790-5791
 * o_proj + residual, :5806-5843 SwiGLU FFN + residual, :5858-5863 output head),
 * each mul_mat_f32 (:465-469) over GGUF Q4_K weights.  Weights: Q4_K blocks
 * (256 weights in 144 bytes: f16 d, f16 dmin, 12 bytes of 6-bit sub-block
 * scales and mins, 128 bytes of 4-bit quants), a row of `cols` weights being
 * cols/256 consecutive blocks; every pointer 16-byte aligned device memory.
 * As in GGML's CPU backend, each activation row is quantised to Q8_K (blocks
 * of 256 int8 with an F32 scale) before the integer dot products.  Calls are
 * ordered on `stream`; on failure they return a status and write a message
 * into err_msg (may be NULL). */

/* y = [residual +] W . x'  or, with w_up, y = silu(W . x') * (W_up . x'),
 * where x' = rms_norm(x) * norm when norm is given (eps inside the root). */
typedef struct hkv_q4k_gemv_args {
    const void *w;          /* Q4_K [rows][cols / 256 blocks]                   */
    const void *w_up;       /* NULL, or the up matrix of a SwiGLU pair (w = gate) */
    int64_t rows;
    int64_t cols;           /* multiple of 256, at most 16384                   */
    int32_t n;              /* activation vectors                               */
    const float *x;         /* [n][cols]                                        */
    const float *norm;      /* NULL or [cols]                                   */
    float eps;
    const float *residual;  /* NULL or [n][rows]; may equal y (in place)         */
    float *y;               /* [n][rows]                                        */
    int32_t tensor_cores;   /* 0: n == 1 on the CUDA cores (dp4a), n > 1 on the
                               tensor cores; 1: tensor cores for every n.  The
                               two sum in different orders (both within 1e-5
                               of GGML's); a backbone created with max_batch
                               > 1 uses 1 throughout                           */
} hkv_q4k_gemv_args;
int hkv_q4k_gemv(const hkv_q4k_gemv_args *args, hkv_stream stream, char *err_msg,
                 size_t err_len);

/* q, k, v projections of x' = rms_norm(x) * norm in one launch, with the
 * per-head rms_norm(.) * q_norm / k_norm of q and k (:5711-5733); RoPE is
 * left to the decode call, which applies it to q and to the appended k. */
typedef struct hkv_q4k_qkv_args {
    const void *wq, *wk, *wv;   /* Q4_K [n_head*128][cols], [n_head_kv*128][cols] x2 */
    int32_t n_head, n_head_kv;
    int64_t cols;
    int32_t n;
    const float *x;             /* [n][cols]                                     */
    const float *norm;          /* NULL or [cols] (attn_norm)                    */
    float eps;
    const float *q_norm;        /* [128]                                         */
    const float *k_norm;        /* [128]                                         */
    float *q_out;               /* [n][n_head*128]                               */
    float *k_out, *v_out;       /* [n][n_head_kv*128]                            */
    int32_t tensor_cores;       /* as in hkv_q4k_gemv_args                       */
} hkv_q4k_qkv_args;
int hkv_q4k_qkv(const hkv_q4k_qkv_args *args, hkv_stream stream, char *err_msg, size_t err_len);

/* Synchronises `stream`; reports (and clears) a bounded device-side wait of a
 * hkv_q4k_gemv / hkv_q4k_qkv launch on the current device that gave up
 * (HKV_ERR_TIMEOUT; the output of that launch is not written). */
int hkv_q4k_sync_check(hkv_stream stream, char *err_msg, size_t err_len);

/* The repo's Q4_K encoder (the reference quantises offline with GGML's tools,
 * scripts/quantize_higgs_gguf_q4_k.py): F32 [rows][cols] -> Q4_K blocks. */
int hkv_q4k_quantize(const float *w, int64_t rows, int64_t cols, void *blocks, hkv_stream stream,
                     char *err_msg, size_t err_len);

/* ------------------------------------------------- backbone decode step -- */
/* A whole decode step of the 36-layer backbone for a batch of slots on one
 * engine: the reference's per-frame graph (run_reference_text_code_frames_
 * backend_kv, :4785-5200, whose per-frame graph is run_kv_decode_graph_all_
 * layers_with_backend_cache_ex, :5629-5863) with the engine's paged KV path
 * in place of the slot cache.  Per layer: hkv_q4k_qkv, hkv_decode_step
 * (RoPE, append, attention), o_proj + residual, SwiGLU FFN + residual; then
 * the output head and greedy codes.  Weights are borrowed (caller-owned). */
typedef struct hkv_backbone hkv_backbone;

typedef struct hkv_backbone_layer {
    const void *attn_q, *attn_k, *attn_v, *attn_output;  /* Q4_K */
    const void *ffn_gate, *ffn_up, *ffn_down;             /* Q4_K */
    const float *attn_norm, *ffn_norm;                     /* [hidden] */
    const float *attn_q_norm, *attn_k_norm;                /* [128]    */
} hkv_backbone_layer;

typedef struct hkv_backbone_weights {
    int32_t hidden;            /* 2560                                          */
    int32_t ffn;               /* 9728                                          */
    int64_t text_vocab;        /* rows of token_embd (151936)                   */
    int32_t n_codebooks;       /* 8   (k_num_codebooks, include/higgs_audio.h:15) */
    int32_t codebook_size;     /* 1026 (k_codebook_vocab_size, :17)            */
    float rms_eps;
    const hkv_backbone_layer *layers; /* host array, one per engine layer       */
    const void *token_embd;    /* Q4_K [text_vocab][hidden]                     */
    const void *audio_embd;    /* Q4_K [n_codebooks*codebook_size][hidden] (a.token_embd) */
    const float *output_norm;  /* [hidden]                                      */
    const void *audio_output;  /* Q4_K [n_codebooks*codebook_size][hidden] (a.output) */
} hkv_backbone_weights;

/* Binds weights to an engine (q/k/v head counts from its config) and
 * allocates activation buffers for up to max_batch slots. */
int hkv_backbone_create(hkv_engine *kv, const hkv_backbone_weights *w, int32_t max_batch,
                        hkv_backbone **out);
void hkv_backbone_destroy(hkv_backbone *bb);
const char *hkv_backbone_last_error(const hkv_backbone *bb);

/* hidden[e] = token_embd[ids[e]] (host ids; text prompt tokens, :2912). */
int hkv_backbone_embed_text(hkv_backbone *bb, int32_t n, const int32_t *ids, hkv_stream stream);
/* hidden[e] = sum over c of a.token_embd[c * codebook_size + codes[e][c]]
 * (:2915-2924, fuse_audio_ids_for_embedding :2546-2562); codes is a DEVICE
 * [n][n_codebooks] array, or NULL for the codes of the last decode. */
int hkv_backbone_embed_codes(hkv_backbone *bb, int32_t n, const int32_t *codes,
                             hkv_stream stream);
/* Runs every layer on hidden[0..n) for slots[e] (appending one row each),
 * advances the slots by one position, and, when want_logits, computes
 * logits = a.output(rms_norm(hidden) * output_norm) and the greedy code of
 * each codebook (the first maximum). */
int hkv_backbone_decode(hkv_backbone *bb, int32_t n, const int32_t *slots, int32_t want_logits,
                        hkv_stream stream);
/* Device buffers: hidden [max_batch][hidden], logits
 * [max_batch][n_codebooks*codebook_size], codes [max_batch][n_codebooks]. */
int hkv_backbone_buffers(const hkv_backbone *bb, float **hidden, float **logits, int32_t **codes);
/* Synchronises `stream` and reports a bad embedding id recorded on the GPU. */
int hkv_backbone_sync_check(hkv_backbone *bb, hkv_stream stream);
/* Kernels this backbone has launched (embedding, projections, argmax; the
 * engine counts the KV path's in hkv_pool_stats.kernel_launches). */
int hkv_backbone_kernel_launches(const hkv_backbone *bb, int64_t *launches);

/* ---------------------------------------------------------- profiling -- */

/* Host time the engine spent inside hkv_decode_step and hkv_decode_attn
 * (entry to return, including the wait for the engine's lock): the calls
 * counted, their total in microseconds, and the part of it that can block on
 * the GPU -- inside the CUDA launch calls (whose queue fills when the host
 * runs far ahead) and waiting to reuse a plan upload buffer still being
 * copied -- since the last reset; reset != 0 clears the counters after
 * reading.  Instrumentation of this engine, no counterpart in the reference:
 * host_us - blocked_us is the engine's own CPU work per call (validation,
 * batch plan), apart from its caller's. */
int hkv_host_stats(hkv_engine *eng, int64_t *calls, double *host_us, double *blocked_us,
                   int reset);

/* When on, every kernel launch is bracketed by CUDA events on its stream;
 * hkv_profile_read synchronises and returns launches and total device ms
 * for one kernel id since the last reset. */
int hkv_profile_enable(hkv_engine *eng, int on);
int hkv_profile_reset(hkv_engine *eng);
int hkv_profile_read(hkv_engine *eng, int kernel_id, int64_t *launches, double *total_ms);

#ifdef __cplusplus
}
#endif

#endif /* HKV_H */
