/*
 * moestream.h -- C ABI of libmoestream.so, the B200 (sm_100a) implementation
 * of moe-stream's per-token MoE expert block and its shared slot pool.
 *
 * Every entry point returns an int status: MS_OK (0) or a negative MS_E_*
 * code; ms_last_error() gives the message of the most recent failure on the
 * calling thread. No C++ exception crosses this boundary. Device buffers are
 * caller-owned and passed as raw pointers plus a CUDA stream (cudaStream_t,
 * passed as void*); the library owns the slot arena, the slot table and its
 * scratch buffers. One host thread at a time may use a pool handle.
 *
 * Reference interfaces each entry point replaces are cited as file:line in
 * the reference repository (agastya-choudhary123/moe-stream).
 */
#ifndef MOESTREAM_H
#define MOESTREAM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------ status codes */
#define MS_OK             0
#define MS_E_INVALID     -1   /* bad argument (ValueError-like)                    */
#define MS_E_CUDA        -2   /* a CUDA call failed                                */
#define MS_E_EXHAUSTED   -3   /* "pool exhausted: every slot pinned or pending"
                                 (engine_v3.py:355-356, RuntimeError)              */
#define MS_E_TIMEOUT     -4   /* a bounded wait ran out                            */
#define MS_E_NOMEM       -5   /* allocation failed                                 */
#define MS_E_STATE       -6   /* call not valid in the handle's current state      */
#define MS_E_IO          -7   /* store read out of range / short (IOError,
                                 engine_v3.py:283-284)                             */
#define MS_E_RANGE       -8   /* an activation (x, or the SwiGLU output h) beyond
                                 the fp16 range (|v| > 65504) reached the fp16
                                 tensor-core operands; that call's output is
                                 not valid                                         */

/* ------------------------------------------------------------- enumerations */
#define MS_MODEL_QWEN3    0   /* engine_v3.py: softmax over E, top-k, renormalise  */
#define MS_MODEL_GPTOSS   1   /* engine_120b.py: top-k logits, softmax over k,
                                 per-projection bias, clamped SwiGLU               */

#define MS_SCALE_BF16     0   /* scales and biases: bf16 [out, in/64] (mx.quantize) */
#define MS_SCALE_FP8      1   /* scales and biases: OCP FP8 E4M3 [out, in/64] times
                                 a per-row 2^(E-127), E one byte per row           */
#define MS_MAX_CLASSES    8

#define MS_EVICT_LFU      0   /* MOE_EVICT=lfu  (engine_v3.py:103, 347-348)        */
#define MS_EVICT_LRU      1   /* MOE_EVICT=lru  (engine_v3.py:345-346)             */
#define MS_EVICT_ASIS     2   /* MOE_EVICT=asis (engine_v3.py:343-344)             */

#define MS_PROJ_GATE      0
#define MS_PROJ_UP        1
#define MS_PROJ_DOWN      2
#define MS_PART_WEIGHT    0   /* U32 [out, in/8]  4-bit codes, low nibble first    */
#define MS_PART_SCALES    1   /* BF16 [out, in/group]                              */
#define MS_PART_BIASES    2   /* BF16 [out, in/group]  (quantisation biases)       */
#define MS_PART_BIAS      3   /* BF16 [out]  gpt-oss projection bias               */

#define MS_MAX_DEPTHS     4

/* ---------------------------------------------------------------- structures */
/* Geometry of one model's expert blobs: experts_index.json (repack.py:137-146,
 * repack_gptoss.py:159-166) plus the model config fields the block reads. */
typedef struct ms_geom {
    int32_t model;            /* MS_MODEL_*                                        */
    int32_t d_model;          /* hidden size (2048 / 2880)                         */
    int32_t d_ff;             /* expert intermediate size (768 / 2880)             */
    int32_t n_experts;        /* experts per layer (128)                           */
    int32_t n_layers;         /* 48 / 36                                           */
    int32_t top_k;            /* 8 / 4                                             */
    int32_t group_size;       /* quantisation group (64)                           */
    int32_t bits;             /* 4                                                 */
    int32_t norm_topk_prob;   /* Qwen3 renormalisation flag                        */
    int32_t proj_bias;        /* 1 if blobs carry the gpt-oss `bias` component     */
    int64_t blob_bytes;       /* padded blob size, a multiple of 16 KiB            */
    int64_t comp_offset[3][4];/* byte offset of [proj][part] in a blob, -1 if none */
} ms_geom;

/* One precision class of expert blobs (ms_pool_set_precision): the codes
 * of a row are a little-endian bit stream of `bits`-bit codes (code j at
 * bit bits*j), rows padded to 16 bytes; scales and biases per group of 64
 * as bf16 or fp8. comp_offset[proj][part], parts: 0 weight, 1 scales,
 * 2 biases, 3 bias (gpt-oss), 4 scales_exp, 5 biases_exp (fp8: one byte per
 * row); -1 where absent. */
typedef struct ms_prec {
    int32_t bits;             /* 2, 3, 4 or 8                                      */
    int32_t scale_fmt;        /* MS_SCALE_*                                        */
    int64_t payload_bytes;    /* bytes of a blob of this class (<= blob_bytes)     */
    int64_t comp_offset[3][6];
} ms_prec;

/* Pool configuration: PF_SLOTS, MOE_EVICT, PF_DEPTH, PF_WIDEN
 * (engine_v3.py:59-62, 84, 103). */
typedef struct ms_pool_config {
    int32_t n_slots;                  /* slots in the HBM arena                    */
    int32_t evict;                    /* MS_EVICT_*                                */
    int32_t n_depths;                 /* entries used in depths[] (0 = no prefetch)*/
    int32_t depths[MS_MAX_DEPTHS];    /* prefetch distances; depths[0] sets the
                                         young-entry window 24*depth (:310-311)    */
    int32_t pf_widen;                 /* speculate top (k * pf_widen) (:84)        */
    int32_t max_tokens;               /* largest T any block call will pass        */
} ms_pool_config;

/* ExpertPool.stats() (engine_v3.py:456-464). Counts, not timings: the
 * reference's blocked/busy_s/depth fields have no device-side equivalent. */
typedef struct ms_stats {
    int64_t total;            /* prefetch + cache + miss                           */
    int64_t prefetch;         /* hits on a slot filled by a prefetch               */
    int64_t cache;            /* true cache hits                                   */
    int64_t miss;             /* demand misses (read on the critical path)         */
    int64_t bail;             /* prefetches abandoned on exhaustion                */
    int64_t issued;           /* prefetch reads issued                             */
    int64_t reads;            /* completed slot fills                              */
    int64_t exposed;          /* demand-miss fills                                 */
    int64_t bytes_read;       /* reads * blob_bytes                                */
    int64_t bytes_exposed;    /* exposed * blob_bytes                              */
} ms_stats;

typedef struct ms_pool ms_pool;

/* ------------------------------------------------------------------ errors */
/* Copies the last error message of this thread into buf (NUL-terminated). */
int ms_last_error(char* buf, size_t n);

/* ---------------------------------------------------------------- the pool */
/* ExpertPool.__init__ (engine_v3.py:128-252): one contiguous HBM arena of
 * n_slots * blob_bytes, slot s at arena + s*blob_bytes, laid out exactly like
 * a store blob, plus the device slot table and scratch for max_tokens. */
int ms_pool_create(const ms_geom* geom, const ms_pool_config* cfg, int device,
                   ms_pool** out);
int ms_pool_destroy(ms_pool* pool);

/* The expert store: (layer, expert) at (layer*n_experts + expert)*blob_bytes
 * (repack.py:141). ms_store_register maps caller memory (pinned or pageable;
 * it is page-locked and mapped for the device); ms_store_alloc allocates
 * mapped pinned memory the pool owns. Replaces the experts.bin fd + preadv
 * worker threads (engine_v3.py:138, 255-301). */
int ms_store_register(ms_pool* pool, void* host, size_t bytes);
int ms_store_alloc(ms_pool* pool, size_t bytes, void** host_out);

/* Router weights of one layer: bf16 [n_experts, d_model] and optional bf16
 * bias [n_experts] (the gate / router Linear the block reads as self.gate /
 * self.router, engine_v3.py:507, engine_120b.py:84). Device pointers. */
int ms_set_router(ms_pool* pool, int layer, const void* w_r, const void* b_r);

/* ExpertPool.prefetch (engine_v3.py:383-396): non-blocking; experts is a
 * host array. Allocation and fills are enqueued on `stream`. */
int ms_pool_prefetch(ms_pool* pool, int layer, const int32_t* experts, int n,
                     void* stream);

/* ExpertPool.acquire (engine_v3.py:398-454): blocking; writes the slot of
 * each expert to the host array slots_out. Returns MS_E_EXHAUSTED when the
 * reference would raise "pool exhausted". */
int ms_pool_acquire(ms_pool* pool, int layer, const int32_t* experts, int n,
                    int32_t* slots_out, void* stream);

/* ExpertPool._read (engine_v3.py:255-290): copy one blob from the store
 * into a slot, bypassing the table (verify_pool.py:200, 212 use it so). */
int ms_pool_read(ms_pool* pool, int slot, int layer, int expert, void* stream);

/* ExpertPool.stats (engine_v3.py:456-464). Synchronises the pool. */
int ms_pool_stats(ms_pool* pool, ms_stats* out);

/* ExpertPool.key_of as layer*n_experts+expert per slot, -1 when empty
 * (engine_v3.py:216). out has n_slots entries. Synchronises the pool. */
int ms_pool_slot_table(ms_pool* pool, int32_t* out);

/* ExpertPool.views[name] base (engine_v3.py:180-194): device address of
 * component [proj][part] of slot 0; slot s is at + s*blob_bytes. */
int ms_pool_component_ptr(ms_pool* pool, int proj, int part, void** out);

/* Whole arena: base address and size in bytes. */
int ms_pool_arena(ms_pool* pool, void** base, size_t* bytes);

/* ------------------------------------------------------------- the block */
/* top_k_experts / top_k_route + top_k_indices (engine_v3.py:467-483,
 * engine_120b.py:65-75) without touching the pool: x bf16 [T, d_model] ->
 * inds int32 [T, top_k], scores bf16 [T, top_k] (descending, exact ties to
 * the lower expert), and, when pred != NULL and layer+depths[0] has a
 * router, pred int32 [T, top_k*pf_widen] for that layer. */
int ms_route(ms_pool* pool, int layer, const void* x, int T, int32_t* inds,
             void* scores, int32_t* pred, void* stream);

/* streaming_call (engine_v3.py:493-609, engine_120b.py:78-149): route,
 * prefetch layer+d for every configured depth, acquire this layer's experts,
 * fill misses from the store, run the 4-bit expert MLPs and the weighted
 * combine. Prefetch fills run on the pool's side stream (ms_pool_join). x, y bf16 [T, d_model] device buffers; T <= max_tokens.
 * Enqueued on `stream`; does not synchronise. Pool exhaustion is reported by
 * the next ms_pool_status / ms_pool_stats call. */
int ms_moe_block(ms_pool* pool, int layer, const void* x, int T, void* y,
                 void* stream);

/* The block fused with its layer's non-expert pieces on either side: the
 * post-attention RMSNorm in front (mlx_lm's Qwen3 / gpt-oss decoder layer:
 * x = rms_norm(h) * norm_w, mx.fast.rms_norm's rounding) and the residual
 * add behind it: out = h + block(x), every value bf16. h is the residual
 * stream (bf16 [T, d_model]), norm_w bf16 [d_model], eps > 0; out may be h.
 * Decode calls of up to 8 tokens normalise inside the route step and add
 * the residual inside the expert kernels' combine (no extra kernel); larger
 * calls normalise with one kernel first. Same asynchronous, capture-safe
 * contract as ms_moe_block. */
int ms_moe_block_fused(ms_pool* pool, int layer, const void* h, const void* norm_w, float eps, int T,
                       void* out, void* stream);

/* Sticky device-side status of asynchronous block calls (MS_OK or the first
 * MS_E_* seen since the last call); clears it. Synchronises `stream`. */
int ms_pool_status(ms_pool* pool, void* stream);

/* No reference counterpart (the reference's prefetch copies are synchronous
 * MLX reads, engine_v3.py:383-396). ms_moe_block copies the slots its
 * prefetches fill on a side stream of the pool, forked after the route step
 * and joined into the stream of the next call that reads the arena (the
 * next block call's expert kernels, ms_expert_mlp, the pool operations).
 * ms_pool_join makes `stream` wait for the fills still pending. Call it on
 * the capturing stream before ending a CUDA graph capture of block calls
 * (the capture must join every stream it forked); the other entry points
 * join by themselves. */
int ms_pool_join(ms_pool* pool, void* stream);

/* kernels.moe_expert_mlp (kernels.py:231-252), generalised to T tokens:
 * slots int32 [T, k] and scores f32 [T, k] (device), x bf16 [T, d_model],
 * y bf16 [T, d_model]. Reads the arena only; no routing, no table.
 * k = top_k with T*k <= MS_MLP_MAX_PAIRS runs the decode kernels; larger
 * batches, and any 1 <= k < top_k, run the grouped tensor-core GEMM (the
 * pool's max_tokens * top_k bounds T*k there). */
int ms_expert_mlp(ms_pool* pool, const int32_t* slots, const float* scores,
                  const void* x, int T, int k, void* y, void* stream);

/* Checkpoint of a pool, no reference counterpart (the reference's pool lives
 * and dies with its process). The state is the slot table with its clocks,
 * counters and statistics and, when with_arena is set, the slot arena
 * itself; a pool restored from a snapshot continues exactly as the saved one
 * did (same slots, same fills, same outputs). ms_pool_state_bytes gives the
 * size of the caller-owned device buffer (256-byte aligned); save and load
 * join the pending prefetch fills into `stream` and enqueue device-to-device
 * copies on it. */
int ms_pool_state_bytes(ms_pool* pool, int with_arena, size_t* bytes);
int ms_pool_save_state(ms_pool* pool, void* dev_buf, int with_arena, void* stream);
int ms_pool_load_state(ms_pool* pool, const void* dev_buf, int with_arena, void* stream);

/* Per-expert precision (the reference's purpose for owning its kernel,
 * kernels.py:25-29, which gather_qmm's single `bits` cannot express): the
 * blob of key (layer, expert) is of class class_of_key[key] (host array of
 * n_layers*n_experts entries) among n_classes classes. The slot and store
 * stride stays geom.blob_bytes (the largest class); a fill copies only its
 * class's payload, and every kernel reads each slot with its class's code
 * width and scale format. Call before any slot is filled (MS_E_STATE
 * after). One class equal to the geometry's own blob restores the default. */
int ms_pool_set_precision(ms_pool* pool, int n_classes, const ms_prec* classes,
                          const uint8_t* class_of_key);

/* Failure-detection self-test, no reference counterpart: enqueues on
 * `stream` one CTA that waits, with the same bounded wait every kernel of the
 * library uses but a limit of limit_ns (at most 2 s), on an mbarrier that
 * never completes. The wait gives up and records MS_E_TIMEOUT in the pool's
 * sticky status, which the next ms_pool_status reports and clears; nothing
 * else changes and the pool stays usable. */
int ms_pool_selftest_wait(ms_pool* pool, long long limit_ns, void* stream);

/* Diagnostic with no reference counterpart: the SASS target the library's
 * kernels carry for `device` (cudaFuncAttributes.binaryVersion of one of
 * them; 100 for sm_100a). */
int ms_kernel_arch(int device, int* binary_version);

/* Device-side routing/slot buffers of the most recent ms_moe_block call
 * (valid until the next call): inds int32 [T,k], scores bf16 [T,k],
 * slots int32 [T,k]. For parity dumps. */
int ms_block_debug(ms_pool* pool, const int32_t** inds, const void** scores,
                   const int32_t** slots);

/* Per-layer CUDA-event timing of ms_moe_block (off by default). When on,
 * every block call records four events on its stream -- before the router,
 * after the router/table step, after the fills and the wait for the previous
 * call's prefetch fills, after the expert kernels -- also inside a CUDA
 * graph capture (they become event nodes). ms_pool_timing reads the last
 * recorded interval of `layer`, in milliseconds: out[0] router+table,
 * out[1] fills (this call's demand fills and the prefetch join), out[2]
 * expert kernels. */
int ms_pool_profile(ms_pool* pool, int enable);
int ms_pool_timing(ms_pool* pool, int layer, float* out3);

/* Expert parallelism (the gpt-oss layer on a 16384-token batch), no counterpart in the reference,
 * which runs on one device; the block it distributes is engine_120b.py:78-149.
 * Each rank holds its experts (and replicas) resident in its pool. The host
 * moves the buffers between ranks
 * (an all-to-all over NCCL) and runs the experts with ms_expert_mlp (k = 1).
 *
 * ms_ep_pack: the T*top_k token/expert pairs of x (routing from ms_route:
 * inds int32 [T, top_k], scores bf16 [T, top_k]) packed destination-major.
 * With placement == NULL expert e goes to rank e / e_local, slot e % e_local.
 * Otherwise placement is a device int32 table [n_experts][1 + 2*max_rep]:
 * the number of replicas of expert e, then (rank, slot) of each replica;
 * pair p = t*top_k + j of expert e goes to replica p % n_rep (replicas of hot
 * experts balance the ranks' loads; every replica computes the same result):
 * send_x bf16 [T*top_k, d_model] (the token's row), send_meta int32
 * [T*top_k][2] (slot on the destination, score as f32 bits), send_counts int32
 * [world] (pairs per destination, device memory), pair_pos int32 [T*top_k]
 * (row of each pair in send_x). Rows inside a destination come in no fixed
 * order. */
int ms_ep_pack(ms_pool* pool, const void* x, int T, const int32_t* inds, const void* scores,
               int world, int e_local, const int32_t* placement, int max_rep, void* send_x,
               int32_t* send_meta, int32_t* send_counts, int32_t* pair_pos, void* stream);

/* ms_ep_combine: y[t] = sum over j of back[pair_pos[t*top_k + j]] (the
 * score-weighted expert outputs returned to their senders), summed in fp32 in
 * j order and rounded once to bf16, as the single-device block does. */
int ms_ep_combine(ms_pool* pool, const void* back, const int32_t* pair_pos, int T, void* y,
                  void* stream);

/* The expert-parallel block through the C ABI alone (no torch.distributed):
 * NCCL is loaded at run time (dlopen of libnccl.so.2, the copy a process
 * already holds if any), so the library needs no NCCL at link time.
 *
 * ms_ep_unique_id: a new NCCL unique id (128 bytes) in out; one rank makes
 * it and the host hands it to every rank by any channel. The calling
 * process runs NCCL's bootstrap root, so it must live until every rank has
 * called ms_ep_init.
 *
 * ms_ep_init: joins this pool (its device, one process or thread per GPU)
 * to a group of `world` ranks; blocks until every rank has joined. The pool
 * holds this rank's experts of the layer resident (ms_pool_read). placement
 * (host int32 [n_experts][1 + 2*max_rep], as ms_ep_pack reads it; NULL for
 * plain sharding: expert e on rank e / (n_experts / world), slot e % that)
 * is copied. MS_E_STATE if the pool already has a group; MS_E_CUDA with the
 * message when NCCL is missing or fails.
 *
 * ms_ep_moe_block: the expert-parallel block on this rank's T tokens x
 * (bf16 [T, d_model], device) -> y (bf16 [T, d_model]), the multi-GPU form
 * of ms_moe_block on `layer` (whose router must be set): route (ms_route),
 * pack (ms_ep_pack), exchange the pair counts and then the rows with NCCL
 * send/recv on `stream`, run the received rows through this rank's experts
 * (ms_expert_mlp, k = 1), send them back and combine (ms_ep_combine). Every
 * rank calls it for the same layer, each with its own T (which may differ);
 * the result equals the single-GPU block bit for bit. One host
 * synchronisation of `stream` per call (the split sizes); the rows a rank
 * receives (up to every rank's T * top_k) must fit the pool's max_tokens.
 * Scratch buffers grow on demand, so the first call at a new size allocates.
 *
 * An exchange that fails or runs past the host wait limit (MS_E_CUDA,
 * MS_E_TIMEOUT: e.g. a rank that died) breaks the group: later calls return
 * MS_E_STATE, and ms_ep_finalize aborts the communicator rather than
 * waiting on its stuck operations.
 *
 * ms_ep_finalize: leaves the group (destroys the communicator, frees the
 * scratch); ms_pool_destroy does it too. */
int ms_ep_unique_id(uint8_t out[128]);
int ms_ep_init(ms_pool* pool, const uint8_t id[128], int rank, int world, const int32_t* placement,
               int max_rep);
int ms_ep_moe_block(ms_pool* pool, int layer, const void* x, int T, void* y, void* stream);
int ms_ep_finalize(ms_pool* pool);

/* ms_expert_mlp without a pool and without any allocation. This entry point
 * has no counterpart in the reference. It is for callers that may not call
 * cudaMalloc when they run the block -- a runtime that reserved all device
 * memory up front and only lends out buffers it planned, an engine whose
 * enqueue step must not allocate -- and so cannot create a pool, whose
 * arena and scratch buffers are allocated. The caller passes the geometry,
 * the expert weights (`arena`: n_slots blobs of geom->blob_bytes, laid out as
 * in the store, e.g. the arena of an existing pool or a caller-owned buffer),
 * slots int32 [T,k], scores f32 [T,k], x bf16 [T,d_model] and y bf16
 * [T,d_model], all device memory on the current device; intermediates live in
 * a fixed ~2 MB __device__ array inside the library, which every GPU that
 * loads the library keeps until the process exits.
 * Limits: T <= MS_STATIC_MAX_TOKENS, T*k <= MS_STATIC_MAX_PAIRS, d_model and
 * d_ff <= 4096 (<= 3072 for gpt-oss), n_slots <= MS_STATIC_MAX_SLOTS; larger
 * sizes, and geometries whose components do not fit in blob_bytes, return
 * MS_E_INVALID before anything is enqueued. A slot index outside
 * [0, n_slots) gives zero rows for its token and is reported by
 * ms_expert_mlp_static_status. The first call on each device looks up the array's device
 * address (cudaGetSymbolAddress); make that first call before any stream
 * capture. All calls share the array: calls that may overlap on the GPU
 * (other streams or host threads) race, so the caller must order them.
 * Enqueued on `stream`; does not synchronise. */
#define MS_STATIC_MAX_TOKENS  16
#define MS_STATIC_MAX_PAIRS   64
#define MS_STATIC_MAX_SLOTS   65536
int ms_expert_mlp_static(const ms_geom* geom, const void* arena, int n_slots,
                         const int32_t* slots, const float* scores, const void* x,
                         int T, int k, void* y, void* stream);

/* Device-side status of the most recent ms_expert_mlp_static call on the
 * current device, which returns before its kernels run: MS_E_INVALID when a
 * slot index was out of range, MS_E_TIMEOUT when a bounded wait for the
 * weight copies ran out, else MS_OK. Waits for `stream`, then clears the
 * status. Allocates nothing either. */
int ms_expert_mlp_static_status(void* stream);

#ifdef __cplusplus
}
#endif
#endif /* MOESTREAM_H */
