// kernels.h -- host-side launchers for the hoard_b200 CUDA kernels (no CUDA types beyond streams).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace hoard {

// Bytes of one GGUF block of 256 weights (Q4_K 144, Q6_K 210), host side.
inline int fmt_block_bytes(int type) { return type == 12 ? 144 : (type == 14 ? 210 : 0); }
inline int64_t fmt_mat_bytes(int type, int64_t n, int64_t k) { return n * (k / 256) * fmt_block_bytes(type); }

// Where one layer's experts live: pool slot s of a layer holds gate | up | down in plane layout at
// base + s*slot_stride + {0, off_up, off_down}. The shared expert (if any) has its own base.
struct LayerWeights {
    const uint8_t* pool;
    int64_t slot_stride;
    int64_t off_up, off_down;
    int n_slots;
    int gate_type, up_type, down_type;
    const uint8_t* shared;        // gate | up | down of the shared expert, or nullptr
    int64_t sh_off_up, sh_off_down;
    int sh_gate_type, sh_up_type, sh_down_type;
    const float* sh_gate_inp;     // [H]
    const float* w_router;        // [E][H]
    const float* w_router_t;      // [H][E] (the persistent decode kernel's per-row router slices)
    const float* w_norm;          // [H]
};

struct Dims {
    int H, E, k, I;
    int renorm;
    float eps;
    int resid_bf16;
    int gemm_ctas;    // CTAs of the tensor-core GEMMs (0 = one per SM); fewer leave SMs to concurrent kernels
};

// Scratch owned by a context (device pointers), sized for max_tokens.
struct Scratch {
    float* fx;        // [T][H]
    int8_t* fx_q;     // [T][H]
    float* fx_d;      // [T][H/256]
    int* fx_bs;       // [T][H/16]
    float* sh_gate;   // [T]
    int32_t* sel;     // [T][k]      (internal routing output when the caller passes none)
    float* w;         // [T][k]
    int* counts;      // [n_slots+1]
    int* offsets;     // [n_slots+2]
    int* perm;        // [T*(k+1)] entry ids (t*KK + j) grouped by slot
    float* h;         // [T*(k+1)][I]
    int8_t* h_q;      // [T*(k+1)][I]
    float* h_d;       // [T*(k+1)][I/256]
    int* h_bs;        // [T*(k+1)][I/16]
    float* y;         // [T*(k+1)][H]
    unsigned* amax;   // [T*(k+1)][I/256] bit patterns of max|h| (persistent decode path)
    float* partials;  // persistent decode: per-CTA partial router sums
    unsigned* sync;   // [0] error bits (1 bad slot id, 2 device wait gave up); persistent decode barrier words
    uint16_t* xq16;   // [T][H] f16 bits: Q8_K-dequantised fx (tensor-core path)
    uint16_t* hq16;   // [T*(k+1)][I] f16 bits: Q8_K-dequantised h in slot-sorted order (tensor-core path)
    int2* items;      // tensor-core work list: (slot, M tile)
    int* n_items;     // [1]
    double* rpart;    // router partial logits per K split
    int* dcount;      // [n_slots+1] dispatch histogram of large batches (zero between calls)
    int* dcursor;     // [n_slots+1] dispatch scatter cursors
};

// Re-lays nrows x nb GGUF blocks of `type` from src (raw) into dst (plane layout).
cudaError_t launch_repack(int type, const uint8_t* src, uint8_t* dst, int64_t nblk_total, cudaStream_t s);
// several matrices re-laid in one launch (every src 16-byte aligned: device or pinned host memory)
constexpr int REPACK_MAX_JOBS = 48;
struct RepackJob {
    int type;
    const uint8_t* src;
    uint8_t* dst;
    int64_t nblk;
};
cudaError_t launch_repack_batch(const RepackJob* jobs, int n, cudaStream_t s);

// dst[c][r] = src[r][c] for an R x C f32 matrix.
cudaError_t launch_transpose(const float* src, float* dst, int R, int C, cudaStream_t s);

// Router: fx, sel, w for T tokens (three launches). `part` holds router_partial_elems() doubles.
int64_t router_partial_elems(int max_tokens, int E);
cudaError_t launch_route(const Dims& d, const LayerWeights& lw, const void* x, int T, float* fx, int32_t* sel,
                         float* w, double* part, cudaStream_t s, int* launches, unsigned* err);

// The grouped expert path for any T (fx given), adding into x_inout.
cudaError_t launch_experts_grouped(const Dims& d, const LayerWeights& lw, const Scratch& sc, const float* fx,
                                   const int32_t* slot_of_sel, const float* w, void* x_inout, int T,
                                   bool need_sh_gate, cudaStream_t s, int* launches, bool prepared = false,
                                   unsigned long long* stamp = nullptr);
// Small batches (T <= 64, H 1024 or 2048, E <= 512), every expert resident: RMSNorm, router logits,
// softmax + top-k, Q8_K of fx and the dispatch with its work list (tile_m entries per item) in one
// kernel; the routing is identical to launch_route's. launch_experts_grouped(..., prepared = true)
// then skips its own quantisation and dispatch.
bool route_fused_supported(const Dims& d, int T);
cudaError_t launch_route_fused(const Dims& d, const LayerWeights& lw, const Scratch& sc, const void* x, int T, int KK,
                               int32_t* sel, float* w, int tile_m, cudaStream_t s, unsigned long long* stamp = nullptr);

// Weight-streaming gate/up and down kernels of the grouped path (persistent, bulk-copy staged; the
// dispatch's work list with one item per non-empty slot). Supported: gate/up Q4_K with H = 2048;
// down Q4_K / Q6_K with I/256 <= 4 and H a multiple of 64.
bool gateup_sw_supported(const Dims& d, const LayerWeights& lw);
bool down_sw_supported(const Dims& d, const LayerWeights& lw);
// stamp: optional {first start, last end} (%globaltimer, atomicMin / atomicMax) of the launch
cudaError_t launch_gateup_sw(const Dims& d, const LayerWeights& lw, const Scratch& sc, int KK, cudaStream_t s,
                             unsigned long long* stamp = nullptr);
cudaError_t launch_down_sw(const Dims& d, const LayerWeights& lw, const Scratch& sc, cudaStream_t s,
                           unsigned long long* stamp = nullptr);

// Pieces shared by the grouped and tensor-core expert paths.
cudaError_t launch_shared_gate(const float* fx, const float* gate_inp, int H, int T, float* out, cudaStream_t s);
// Counting sort of the entries by slot; with tile_m > 0 also the (slot, M tile) work list. Slots out
// of range set error bit 1 and are skipped; with skip_neg, negative slots are skipped silently (the
// unused rows of the expert-parallel receive regions).
cudaError_t launch_dispatch(const int32_t* slot_of_sel, int T, int k, int KK, int n_slots, const Scratch& sc,
                            int tile_m, cudaStream_t s, int* launches, bool skip_neg = false);
// y_half: sc.y holds f16 rows (tensor-core path) instead of f32 rows (grouped path)
cudaError_t launch_combine(const Dims& d, const Scratch& sc, const float* w, void* x_inout, int T, int KK,
                           cudaStream_t s, bool y_half);

// The tensor-core grouped GEMM expert path (prefill / batched tokens), adding into x_inout.
bool tc_supported(const Dims& d, const LayerWeights& lw);
// Router logits of large batches on the tensor cores (tf32 with a hi/lo split, f32-accurate): partial
// sums of `ksplit` K ranges into part[ksplit][T][E] (double), the layout k_route_topk sums.
cudaError_t launch_router_tc(const float* fx, const float* w_router, int T, int H, int E, int ksplit, double* part,
                             unsigned* err, cudaStream_t s);
int64_t tc_max_items(int T, int KK, int n_slots);
int64_t tc_trace_elems();   // stamps written by one call when tracing: [gate/up, down][cta][item][stage][slot]
cudaError_t launch_experts_tc(const Dims& d, const LayerWeights& lw, const Scratch& sc, const float* fx,
                              const int32_t* slot_of_sel, const float* w, void* x_inout, int T, cudaStream_t s,
                              int* launches, unsigned long long* trace);

// Expert parallelism: the experts of R already-quantised rows, each bound to a slot, into y_out [R][H];
// the combine of rows that came back in send order (pos[t*k + j] = row of entry (t, j)); the f16
// Q8_K rows of fx; the pack of (token, j) entries by destination rank.
cudaError_t launch_experts_tc_rows(const Dims& d, const LayerWeights& lw, const Scratch& sc, const uint16_t* rows,
                                   const int32_t* slot_of_row, int R, uint16_t* y_out, cudaStream_t s, int* launches);
cudaError_t launch_combine_rows(const Dims& d, const uint16_t* y, const int* pos, const float* w, void* x_inout, int T,
                                cudaStream_t s);
cudaError_t launch_q8_rows(const float* fx, int T, int H, uint16_t* out, cudaStream_t s);
cudaError_t launch_ep_pack(const int32_t* sel, int T, int k, int n_ranks, int experts_per_rank, const uint16_t* xq,
                           int H, int* counts, int* cursor, int* pos_of_entry, int32_t* send_expert,
                           uint16_t* send_rows, unsigned* err, cudaStream_t s, int* launches);

// ---- per-token operations of a decode step around the MoE layers (kernels_harness.cu) ----
cudaError_t launch_rmsnorm_f32(const float* x, int rows, int cols, float eps, const float* w, float* out,
                               cudaStream_t s);
cudaError_t launch_quant_q8(const float* x, int rows, int K, int8_t* q, float* d, int* bs, cudaStream_t s);
cudaError_t launch_embed(int type, const uint8_t* table, int H, int64_t n_vocab, const int32_t* token,
                         const int32_t* pos, float* out, cudaStream_t s);
cudaError_t launch_qgemv(int type, const uint8_t* w, int N, int K, const int8_t* xq, const float* xd, const int* xbs,
                         const float* resid, float* y, cudaStream_t s);
// KV caches hold f16, or bf16 when kv_bf16
cudaError_t launch_rope_store(float* q, float* k, const float* v, int n_head, int n_kv, int hd, int pos,
                              const int32_t* pos_dev, int max_ctx, float freq_base, void* kc, void* vc, bool kv_bf16,
                              cudaStream_t s);
size_t attention_smem(int hd, int n_pos);
cudaError_t launch_attention(const float* q, const void* kc, const void* vc, bool kv_bf16, int n_head, int n_kv,
                             int hd, int n_pos, const int32_t* pos_dev, float scale, const float* gate, int gstride,
                             float* out, cudaStream_t s);
cudaError_t launch_argmax(const float* v, int n, int32_t* out, int32_t* pos, int seq_len, cudaStream_t s);
cudaError_t launch_rmsnorm_q8(const float* x, int H, float eps, const float* w, int8_t* q, float* d, int* bs,
                              cudaStream_t s);
cudaError_t launch_qgemv_set(int n, const int* types, const uint8_t* const* w, const int* N, int K,
                             const float* const* resid, float* const* y, const int8_t* xq, const float* xd,
                             const int* xbs, cudaStream_t s);
cudaError_t launch_qknorm_rope_store(const float* q, const float* k, const float* v, const float* qn, const float* kn,
                                     int mode, float eps, int n_head, int n_kv, int hd, int q_stride, int rope_dim,
                                     int pos, const int32_t* pos_dev, int max_ctx, float freq_base, float* q_out,
                                     void* kc, void* vc, bool kv_bf16, cudaStream_t s);
// Gated delta-net decode step of one token (d_state 128): causal conv over a ring of the last d_conv
// inputs, the delta-rule state update and the gated RMSNorm; see kernels_harness.cu
cudaError_t launch_gdn_step(const float* qkv, const float* z, const float* ba, const float* conv_w, float* ring,
                            const float* dt_bias, const float* ssm_a, const float* norm_w, float* state, int Hv, int Hk,
                            int d_state, int d_conv, float eps, int pos, const int32_t* pos_dev, float* out,
                            cudaStream_t s);

// ---- expert parallelism over NVLink peer memory ----
// Every rank allocates one block with this layout (identical on all ranks, so a peer's field is its
// base + the same offset); peers map it (CUDA IPC) and write into it directly.
//   flags[64]   u32  barrier epochs, flags[s] written by rank s
//   count[64]   i32  count[s]: rows rank s sent here this layer
//   start[64]   i32  start[s]: where those rows begin in rank s's send order
//   expert      i32  [G][cap] expert id of each received entry, region s written by rank s
//   row_of      i32  [G][cap] the entry's token row within region s of `rows`
//   rows        f16  [G][cap_rows][H] received Q8_K-dequantised token rows, one per (token, this rank)
//                    however many of the token's experts this rank computes; region s written by rank s
//   yback       f16  [cap][H] expert outputs of this rank's own entries, in its send order, written by
//                    the ranks that computed them
struct P2PLayout {
    int64_t flags, count, start, expert, row_of, rows, yback, bytes;
};
P2PLayout p2p_layout(int G, int cap, int cap_rows, int H);

struct P2PSend {
    uint8_t* const* peer;    // device [G] block base of every rank (own included)
    P2PLayout L;
    int G, rank, cap, cap_rows, H, epr;
};
// Send side of one layer: entries counted by destination rank, their starts and counts written into
// every destination's count/start[rank], pos_of_entry[e] = the entry's send position, each entry's
// expert id and token row written into the destination's region `rank`, and each token's f16 row
// written once per destination rank that computes any of its experts (rowinfo[e] >= 0 marks the entry
// that sends it; rcursor counts rows per destination).
cudaError_t launch_p2p_send(const P2PSend& p, const int32_t* sel, int T, int k, const uint16_t* xq, int* counts,
                            int* cursor, int* start, int* rcursor, int* pos_of_entry, int* rowinfo, unsigned* err,
                            cudaStream_t s, int* launches);
// Barrier halves: signal writes `epoch` into every rank's flags[rank] (system-scope release after a
// system fence); wait spins (bounded by timeout_ns, then error bit 2) until every flags[s] >= epoch.
// A wait returns at once when bit 2 is already set.
cudaError_t launch_p2p_signal(const P2PSend& p, uint32_t epoch, cudaStream_t s);
cudaError_t launch_p2p_wait(const uint8_t* block, const P2PLayout& L, int G, uint32_t epoch,
                            unsigned long long timeout_ns, unsigned* err, cudaStream_t s);
// Receive side: slot of every region entry (-1 for the unused tail of a region, and for every entry
// when error bit 2 is set) and its activation row (arow), then the tensor-core FFN whose down
// epilogue stores y of region entry (s, i) into rank s's yback[start[s] + i].
cudaError_t launch_p2p_experts(const Dims& d, const LayerWeights& lw, const Scratch& sc, const P2PSend& p,
                               const uint8_t* block, int slot_base, int* slots, int* arow, cudaStream_t s,
                               int* launches);

// Persistent fused decode kernel over n_layers layers (T <= decode_max_tokens()).
int decode_max_tokens();
int decode_grid();           // CTAs of a persistent launch (one per SM)
int decode_trace_phases();   // stamps per CTA and layer written when tracing
bool decode_supported(const Dims& d, const LayerWeights* lws, int n_layers);
// KK: expert positions (d.k, plus 1 when the layers have a shared expert); sh_dt: its down type
cudaError_t launch_decode_persistent(const Dims& d, int KK, int sh_dt, const LayerWeights* lws_dev, int n_layers,
                                     const Scratch& sc, void* x_inout, int T, int32_t* sel_out, float* w_out,
                                     cudaStream_t s, unsigned long long* trace);

// The same persistent decode kernel with its scratch in a static device array (no allocation).
// scratch: the array's device address on the current device, from decode_static_address
bool decode_static_fits(const Dims& d, int KK);
cudaError_t decode_static_address(void** out);
// byte offset of the static scratch's error word (the same bits as Scratch::sync[0])
size_t decode_static_error_offset();
cudaError_t launch_decode_static(const Dims& d, int KK, int sh_dt, const LayerWeights* lws_dev, int n_layers,
                                 void* scratch, void* x_inout, int32_t* sel_out, float* w_out, cudaStream_t s);

}  // namespace hoard
