/* hoard_moe.h -- C ABI of the B200-native MoE layer (router -> expert dispatch -> SwiGLU expert
 * FFN on Q4_K/Q6_K -> weighted combine into the residual).
 *
 * This is the boundary that hoard's C++ layer schedule calls in place of its inline ggml graph
 * code for one MoE layer. Each entry point names the hoard code it replaces (paths inside the
 * hoard project). Conventions, for every function:
 *   - returns HOARD_OK (0) or a negative HOARD_E* status; never exits, never throws;
 *   - device buffers passed in are owned by the caller; the context owns its expert pool,
 *     router weights and scratch;
 *   - one context is driven by one host thread at a time;
 *   - a stream argument of NULL means the legacy default stream.
 */
#ifndef HOARD_MOE_H
#define HOARD_MOE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define HOARD_OK 0
#define HOARD_EINVAL (-1)   /* bad argument: size, type, index, null pointer */
#define HOARD_ENOMEM (-2)   /* device or pinned-host allocation failed */
#define HOARD_ECUDA (-3)    /* a CUDA runtime call failed; see hoard_moe_last_error */
#define HOARD_ETIMEOUT (-4) /* a bounded device-side wait gave up */
#define HOARD_ENCCL (-5)    /* a collective failed */
#define HOARD_ESTATE (-6)   /* call out of order, e.g. experts before any route on this context */

/* weight / activation types: GGUF (ggml) type ids */
#define HOARD_TYPE_F32 0
#define HOARD_TYPE_F16 1
#define HOARD_TYPE_Q4_K 12
#define HOARD_TYPE_Q6_K 14
#define HOARD_TYPE_BF16 30

typedef struct hoard_moe_ctx hoard_moe_ctx;
typedef void* hoard_stream; /* a cudaStream_t */

/* Layer hyper-parameters. hoard reads these from GGUF metadata in load_model
 * (src/run_moe_stream.cpp:125-151; src/run_qwen35.cpp:160-200). */
typedef struct hoard_moe_desc {
    int n_embd;          /* H: hidden size (multiple of 256) */
    int n_expert;        /* E: experts per layer (<= 1024) */
    int n_expert_used;   /* k: experts per token (<= 16); the TOPK override of
                            src/run_qwen35.cpp:169 is expressed by passing a smaller k */
    int n_ff;            /* I: expert intermediate size (multiple of 256) */
    int n_layer;         /* layers held by this context */
    int n_slots;         /* expert slots per layer; n_expert = all experts HBM-resident */
    int norm_topk;       /* 1: renormalise the top-k weights to sum 1 (clamped at
                            6.103515625e-5), src/run_moe_stream.cpp:150, :371-373 */
    float eps;           /* RMSNorm epsilon */
    int resid_type;      /* HOARD_TYPE_F32 or HOARD_TYPE_BF16: dtype of x / x_inout */
    const int* gate_types; /* [n_layer] HOARD_TYPE_Q4_K / _Q6_K, or NULL = all Q4_K */
    const int* up_types;   /* [n_layer] or NULL = all Q4_K */
    const int* down_types; /* [n_layer] or NULL = all Q6_K (per-layer mix: H.dtype[il],
                              src/run_moe_stream.cpp:179) */
    int n_ff_shexp;      /* shared-expert intermediate size; 0 = none. Must equal n_ff when set
                            (src/run_qwen35.cpp:195, :659-666) */
    int shexp_gate_type; /* types of the shared expert's gate/up/down */
    int shexp_up_type;
    int shexp_down_type;
    int max_tokens;      /* largest T of any call (sizes the scratch) */
    int device;          /* CUDA device ordinal */
} hoard_moe_desc;

/* Creates a context: allocates the HBM expert pool [n_layer][n_slots] and the scratch.
 * Replaces the slot-pool allocation of src/run_moe_stream.cpp:242-254. */
int hoard_moe_create(const hoard_moe_desc* desc, hoard_moe_ctx** out);

/* Frees everything the context owns. */
int hoard_moe_destroy(hoard_moe_ctx* ctx);

/* Sets one layer's router weight ffn_gate_inp (f32 [E][H]: GGUF ne=[H,E]) and its ffn_norm
 * (f32 [H]). Host or device pointers. Replaces the resident tensors read by
 * src/run_moe_stream.cpp:352-353. */
int hoard_moe_set_router(hoard_moe_ctx* ctx, int layer, const float* w_router, const float* w_norm);

/* Copies one expert's raw GGUF block bytes (gate [I][H], up [I][H], down [H][I], each in the
 * layer's type, per-expert stride as stored in the GGUF file) into pool slot `slot` of
 * `layer`, asynchronously on `stream`. Host (pinned for true asynchrony) or device pointers.
 * The bytes are re-laid into the pool's plane layout on the device.
 * Replaces to_vram (src/run_moe_stream.cpp:279-284) and the pool upload in ensure
 * (src/run_specloop.cpp:63-65). */
int hoard_moe_upload_expert(hoard_moe_ctx* ctx, int layer, int slot, const void* gate,
                            const void* up, const void* down, hoard_stream stream);

/* Sets one layer's shared expert (raw GGUF bytes of ffn_{gate,up,down}_shexp) and its gate
 * vector ffn_gate_inp_shexp (f32 [H]). Replaces src/run_qwen35.cpp:659-666's resident tensors. */
int hoard_moe_set_shared(hoard_moe_ctx* ctx, int layer, const void* gate, const void* up,
                         const void* down, const float* gate_inp);

/* Router for T tokens: fx = rms_norm(x) * ffn_norm; probs = softmax(W_r . fx) over all E;
 * sel = top-k (descending, ties to the lower id); w = probs[sel], renormalised if norm_topk.
 * x: device [T][H] of resid_type. sel [T][k] int32 and w [T][k] f32: device or pinned host.
 * fx is kept in the context for the next hoard_moe_experts call.
 * Replaces graph A's router tail + readback + renorm, src/run_moe_stream.cpp:352-373. */
int hoard_moe_route(hoard_moe_ctx* ctx, int layer, const void* x, int T, int32_t* sel, float* w,
                    hoard_stream stream);

/* Expert FFN + weighted combine: x_inout[t] += sum_j w[t][j] * FFN_{slot(t,j)}(fx[t])
 * (+ the gated shared expert). fx: device f32 [T][H], or NULL to use the fx of the last
 * hoard_moe_route on this context. sel [T][k]: expert ids; slot_of_sel [T][k]: pool slots, or
 * NULL when slot == expert id (all experts resident). Device pointers.
 * Replaces graph B + the host weighted sum, src/run_moe_stream.cpp:425-447, and the batched
 * mul_mat_id form src/run_specloop.cpp:125-140. */
int hoard_moe_experts(hoard_moe_ctx* ctx, int layer, const float* fx, const int32_t* sel,
                      const int32_t* slot_of_sel, const float* w, void* x_inout, int T,
                      hoard_stream stream);

/* Fused layer with every expert resident (slot == expert id): route + experts + combine, with
 * no host round trip. sel_out / w_out may be NULL. For 2 <= T <= 64 below the GEMM threshold the
 * RMSNorm, router, top-k, Q8_K of fx and dispatch run as one kernel whose routing is bit-for-bit
 * that of hoard_moe_route. Replaces src/run_moe_stream.cpp:352-447 for the all-resident case
 * (K = n_expert) and the fused chain of src/run_m1.cpp:92-108. */
int hoard_moe_layer(hoard_moe_ctx* ctx, int layer, void* x_inout, int T, int32_t* sel_out,
                    float* w_out, hoard_stream stream);

/* n_layers consecutive fused layers [layer0, layer0 + n_layers) on the same x_inout (an MoE
 * stack with nothing between the layers). sel_out / w_out, if given, are [n_layers][T][k]. */
int hoard_moe_layers(hoard_moe_ctx* ctx, int layer0, int n_layers, void* x_inout, int T,
                     int32_t* sel_out, float* w_out, hoard_stream stream);

/* Decode (T = 1) through n_layers consecutive fused layers, like hoard_moe_layers, but without any
 * device allocation and without the context's scratch: the kernel's scratch (about 105 KiB) is a
 * fixed device array inside this library. It exists for callers that cannot allocate device memory
 * when they run a step: an engine whose device memory is entirely handed out by its own arena after
 * start-up (hoard sizes its expert slot pool to the whole VRAM budget), or a step loop that must not
 * call cudaMalloc at all (it can synchronise the device, and a failure mid-step has no recovery).
 * The weights stay in a context created at start-up. No counterpart in the hoard project.
 *   - Limits: n_expert_used (plus 1 with a shared expert) <= 16, n_ff <= 1024, n_expert <= 512;
 *     larger shapes return HOARD_EINVAL. Contexts the persistent decode kernel cannot serve return
 *     HOARD_ESTATE.
 *   - hoard_moe_create looks up the array's device address (cudaGetSymbolAddress) on the context's
 *     device, which also loads the code module that holds the array: the array is reserved when the
 *     context is created, before the caller's arena takes the rest of the device memory. A context
 *     must not be used across a device reset (cudaDeviceReset), which invalidates that address.
 *   - Every call on a device shares the one array; each call clears the parts that must start at
 *     zero. Calls whose kernels overlap on the GPU (other streams, other threads) race: serialise them.
 *   - Device-side errors (an id out of range, a wait that gave up) go to the static array's own error
 *     word, which the next call clears: read it with hoard_moe_decode_noalloc_status after a call.
 * x_inout: device [H] of resid_type; sel_out / w_out: NULL or [n_layers][k]. */
int hoard_moe_decode_noalloc(hoard_moe_ctx* ctx, int layer0, int n_layers, void* x_inout, int32_t* sel_out,
                             float* w_out, hoard_stream stream);
/* Waits for `stream`, then reports and clears the error word of the static decode scratch (the
 * statuses of hoard_moe_sync_status); allocates nothing. */
int hoard_moe_decode_noalloc_status(hoard_moe_ctx* ctx, hoard_stream stream);

/* Waits for `stream`, then reports and clears the errors kernels recorded on the device:
 * HOARD_EINVAL for expert or slot ids out of range (those entries were skipped), HOARD_ETIMEOUT
 * for a bounded device-side wait that gave up. hoard aborts on such input instead
 * (src/run_moe_stream.cpp:56); this library reports it. */
int hoard_moe_sync_status(hoard_moe_ctx* ctx, hoard_stream stream);

/* Phase tracing of the persistent decode kernel (the counterpart of hoard's per-phase timers
 * tA/tFetch/tB, src/run_qwen35.cpp:434-435, :846-853). With capacity > 0, every later T = 1 fused
 * launch whose stamps fit writes %globaltimer values (ns) into dev_buf laid out
 * [cta][layer][phase]; capacity 0 turns tracing off. Phases: 0 layer start, 1 routed,
 * 2 copies issued, 3 fx quantised, 4 gate/up bytes landed, 5 h written, 6 past barrier,
 * 7 h quantised, 8 down bytes landed, 9 down done, 10 combined + router sums, 11 past barrier.
 * The tensor-core expert path (T >= the GEMM threshold) writes, when capacity >= 4096, stamps
 * [gemm: gate/up, down][cta < 4][item < 2][stage < 32][8]: 0 stage full at the MMA thread,
 * 1 committed, 2 B-row 0 dequant start, 3 B-row 0 saw the stage empty, 4 B-row 0 arrived,
 * 5 A-thread 0 saw the stage empty, 6 A-thread 0 issued; slot 7 of stages 0/1 = epilogue
 * start/end. The small-batch layer path (2 <= T <= 64, every expert resident) writes, when
 * capacity >= 6, {first start, last end} pairs of its fused route, gate/up and down kernels into
 * words 0-5 by atomicMin / atomicMax: the caller sets the starts to UINT64_MAX and the ends to 0. */
int hoard_moe_set_trace(hoard_moe_ctx* ctx, uint64_t* dev_buf, int64_t capacity);

/* CTAs per persistent launch and stamps per (CTA, layer) of the trace layout. */
int hoard_moe_trace_layout(const hoard_moe_ctx* ctx, int* ctas, int* phases);

/* Bytes of one expert's raw GGUF gate+up+down at `layer` (what upload_expert reads). */
int64_t hoard_moe_expert_bytes(const hoard_moe_ctx* ctx, int layer);

/* Kernel launches issued by this context since creation (instrumentation). */
int64_t hoard_moe_launch_count(const hoard_moe_ctx* ctx);

/* Selects the decode implementation for small T: 0 = grouped kernels (any T),
 * 1 = persistent fused decode kernel (default where supported). */
int hoard_moe_set_decode_impl(hoard_moe_ctx* ctx, int impl);

/* Token count at or above which hoard_moe_experts / hoard_moe_layer(s) run the expert FFN as the
 * token-sorted grouped GEMM on the tensor cores (weights dequantised to f16 in shared memory, f32
 * accumulation) instead of the exact-integer grouped kernels; 0 = never. Default 96 (C2 shape, measured:
 * the weight-streaming kernels take 259 / 348 / 439 us at T = 64 / 96 / 128, the tensor-core path a
 * flat ~345-356 us from T = 64 to 256: they cross at T ~ 96). The batched
 * counterpart of hoard's mul_mat_id path (src/run_specloop.cpp:125-140); hoard has no such switch,
 * its graph picks the backend's matmul kernel by batch size. */
int hoard_moe_set_gemm_min_tokens(hoard_moe_ctx* ctx, int min_tokens);

/* CTAs of the tensor-core GEMM launches (0 = one per SM, the default). Fewer leave SMs free for
 * kernels that should run alongside, e.g. NCCL's all-to-all of the next micro-batch during expert
 * parallelism (hoard_b200/ep.py). No counterpart in hoard. */
int hoard_moe_set_gemm_ctas(hoard_moe_ctx* ctx, int ctas);

/* Top-k override (hoard's TOPK, src/run_qwen35.cpp:169): route, experts and layer calls from now on
 * select k experts per token, 1 <= k <= the n_expert_used the context was created with (its buffers
 * are sized for that). Renormalisation follows norm_topk over the k selected. */
int hoard_moe_set_top_k(hoard_moe_ctx* ctx, int k);

/* ---- Residency: per-layer LRU slot pool over a host RAM tier --------------------------------------
 * Replaces hoard's to_vram / fetch and its per-layer LRU (src/run_moe_stream.cpp:279-284, :380-421;
 * the `ensure` of src/run_specloop.cpp:123) when n_slots < n_expert. Uploads run on the context's own
 * upload stream (raw GGUF bytes H2D, re-laid into the slot); the compute stream waits only for the
 * uploads of the slots a call uses, and a slot is overwritten only after the last hoard_moe_experts
 * call of its layer that may read it. */

/* Registers the host copy (raw GGUF bytes, as hoard_moe_upload_expert takes them) of one expert. The
 * caller keeps the memory alive. Page-locked (or device) memory whose three matrices start on 16-byte
 * boundaries is read in place by the re-lay kernel over PCIe (no staging copy; all misses of one
 * hoard_moe_ensure call in one launch); pageable memory goes through a staging buffer. */
int hoard_moe_ram_tier(hoard_moe_ctx* ctx, int layer, int expert, const void* gate, const void* up,
                       const void* down);

/* For n selected expert ids (host array, e.g. the routed sel of one token), returns their pool slots in
 * slot_of_sel (host array), uploading misses from the RAM tier into least-recently-used slots that this
 * call does not use, and makes `stream` wait for those uploads. Pass the slots (copied to the device)
 * to hoard_moe_experts on the same stream. HOARD_EINVAL if one call needs more slots than n_slots,
 * HOARD_ESTATE if a selected expert was never registered with hoard_moe_ram_tier. */
int hoard_moe_ensure(hoard_moe_ctx* ctx, int layer, const int32_t* sel, int n, int32_t* slot_of_sel,
                     hoard_stream stream);

/* Lookups that hit / missed and raw bytes uploaded by hoard_moe_ensure since creation (hoard's
 * 3-tier metrics, src/run_moe_stream.cpp:539-543). */
int hoard_moe_residency_stats(const hoard_moe_ctx* ctx, int64_t* hits, int64_t* misses, int64_t* bytes_uploaded);

/* ---- Expert parallelism (batched tokens over G ranks, experts [g*E/G, (g+1)*E/G) on rank g) ----
 * The sharded counterpart of the single-process mul_mat_id of src/run_specloop.cpp:125-140, which
 * hoard runs on one GPU only. One context per rank; its pool holds at least the rank's own experts.
 * Per layer: hoard_moe_route -> hoard_moe_ep_pack -> all-to-all of send_counts, then of send_rows and
 * send_expert (rows for rank r are the r-th run of send_counts) -> hoard_moe_ep_experts on the
 * received rows -> all-to-all of y back (the reverse splits) -> hoard_moe_ep_combine. The exchange is
 * the caller's (NCCL / torch.distributed); every row is computed independently and y travels in the
 * same f16 form the single-rank tensor-core path stores, so G ranks reproduce it bit for bit. */

/* Reserves the receive-side scratch for up to max_rows rows per hoard_moe_ep_experts call. */
int hoard_moe_ep_reserve(hoard_moe_ctx* ctx, int64_t max_rows);

/* Send side, after hoard_moe_route(ctx, layer, x, T, sel, w) on the same stream: counting-sorts the
 * T*k (token, j) entries by destination rank sel / experts_per_rank and gathers their Q8_K-quantised
 * activation rows (q*d as f16). Device outputs: send_counts [n_ranks] rows per destination, in rank
 * order; pos_of_entry [T*k] the send row of entry t*k+j (-1 if its expert id was out of range:
 * reported by hoard_moe_sync_status); send_expert [T*k] the global expert id of each send row;
 * send_rows [T*k][n_embd] f16 bits. Within one destination the row order is unspecified. */
int hoard_moe_ep_pack(hoard_moe_ctx* ctx, int layer, const int32_t* sel, int T, int n_ranks,
                      int experts_per_rank, int32_t* send_counts, int32_t* pos_of_entry, int32_t* send_expert,
                      uint16_t* send_rows, hoard_stream stream);

/* Receive side: expert FFN (gate/up, SwiGLU, Q8_K of h, down) of R received rows (f16 [R][n_embd])
 * bound to this context's pool slots slot_of_row [R], into y_out [R][n_embd] f16 bits (device
 * pointers; values clamped to the f16 range). R <= the reserved max_rows. */
int hoard_moe_ep_experts(hoard_moe_ctx* ctx, int layer, const uint16_t* rows, const int32_t* slot_of_row, int R,
                         uint16_t* y_out, hoard_stream stream);

/* Send side: x[t] += sum_j w[t][j] * y_back[pos_of_entry[t*k+j]] (j ascending, the combine of
 * src/run_moe_stream.cpp:447), y_back [T*k][n_embd] f16 bits in send order. */
int hoard_moe_ep_combine(hoard_moe_ctx* ctx, const float* w, const int32_t* pos_of_entry, const uint16_t* y_back,
                         void* x_inout, int T, hoard_stream stream);

/* ---- Expert parallelism over NVLink peer memory (no host round trip, no collective library) ----
 * The same sharding as above, with the exchange done by this library's own kernels: every rank owns
 * one symmetric block (per source rank: the received entries' expert ids and token rows [cap],
 * cap = max_tokens * k, and the token rows [max_tokens][n_embd] f16; the per-source counts; and
 * y_back [cap][n_embd]) that all ranks map. Per layer, on each rank's stream:
 *   hoard_moe_p2p_send    route; entries counted by destination; expert ids stored straight into each
 *                         destination's region `rank`, and each token row once per destination rank
 *                         that computes any of its experts; signal
 *   hoard_moe_p2p_compute wait for every rank's send; expert FFN (tensor cores) of the received rows,
 *                         the down epilogue storing each output row straight into its source rank's
 *                         y_back; signal
 *   hoard_moe_p2p_finish  wait for every rank's compute; x[t] += sum_j w_j y_back[pos(t, j)]
 * Waits are bounded (hoard_moe_p2p_set_timeout, default 5 s): on expiry they set the error that
 * hoard_moe_sync_status reports as HOARD_ETIMEOUT, later waits return at once and the received rows
 * are skipped, so the context stays usable; the peer group must then be closed and re-opened on every
 * rank. Results equal hoard_moe_layer's on one GPU bit for bit. Layers with a shared expert are not
 * supported (HOARD_EINVAL). */
#define HOARD_P2P_HANDLE_BYTES 128

/* Allocates this rank's block (zeroed) and the receive-side scratch. The rank computes experts
 * [rank*experts_per_rank, (rank+1)*experts_per_rank) held in pool slots slot_base... */
int hoard_moe_p2p_init(hoard_moe_ctx* ctx, int n_ranks, int rank, int experts_per_rank, int slot_base);

/* HOARD_P2P_HANDLE_BYTES describing this rank's block (a CUDA IPC handle plus the layout), to be
 * all-gathered by the caller. */
int hoard_moe_p2p_handle(hoard_moe_ctx* ctx, void* handle_out);

/* Maps every other rank's block from the all-gathered handles ([n_ranks][HOARD_P2P_HANDLE_BYTES],
 * rank order; processes of one node). */
int hoard_moe_p2p_open(hoard_moe_ctx* ctx, const void* handles);

/* The same for ranks that are contexts of this process (peers[n_ranks], peers[rank] == ctx; on the same
 * or on other GPUs of the node). */
int hoard_moe_p2p_attach(hoard_moe_ctx* ctx, hoard_moe_ctx* const* peers);

/* Unmaps the peers' blocks and resets this rank's barrier state; every rank closes before any re-opens. */
int hoard_moe_p2p_close(hoard_moe_ctx* ctx);

int hoard_moe_p2p_set_timeout(hoard_moe_ctx* ctx, double seconds);

/* The three steps of one layer (above); x [T][n_embd] on this rank, T <= max_tokens (ranks may differ).
 * sel_out / w_out may be null (internal buffers); w must stay valid until hoard_moe_p2p_finish. */
int hoard_moe_p2p_send(hoard_moe_ctx* ctx, int layer, const void* x, int T, int32_t* sel_out, float* w_out,
                       hoard_stream stream);
int hoard_moe_p2p_compute(hoard_moe_ctx* ctx, hoard_stream stream);
int hoard_moe_p2p_finish(hoard_moe_ctx* ctx, void* x_inout, hoard_stream stream);

/* send + compute + finish over layers [layer0, layer0 + n_layers); sel_out / w_out as in
 * hoard_moe_layers ([n_layers][T][k] or null). */
int hoard_moe_p2p_layers(hoard_moe_ctx* ctx, int layer0, int n_layers, void* x_inout, int T, int32_t* sel_out,
                         float* w_out, hoard_stream stream);

/* Last error message of this context (CUDA error string or argument check). */
const char* hoard_moe_last_error(const hoard_moe_ctx* ctx);

/* Static description of a status code. */
const char* hoard_strerror(int status);

#ifdef __cplusplus
}
#endif

#endif /* HOARD_MOE_H */
