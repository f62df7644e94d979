// moe_api.cpp -- the C ABI of include/hoard_moe.h: context, HBM expert pool, router weights,
// scratch, uploads and the per-call dispatch between the persistent decode kernel and the grouped
// path. Host C++ only; kernels are launched through kernels.h.
#include "../../include/hoard_moe.h"
#include "kernels.h"

#include <cuda_runtime.h>
#include <algorithm>
#include <array>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

using namespace hoard;

namespace {

constexpr int64_t kAlign = 256;
inline int64_t align_up(int64_t v) { return (v + kAlign - 1) / kAlign * kAlign; }
inline bool is_quant(int t) { return t == HOARD_TYPE_Q4_K || t == HOARD_TYPE_Q6_K; }

struct LayerStore {
    int gt = HOARD_TYPE_Q4_K, ut = HOARD_TYPE_Q4_K, dt = HOARD_TYPE_Q6_K;
    int64_t gate_bytes = 0, up_bytes = 0, down_bytes = 0;   // raw GGUF bytes per expert
    int64_t off_up = 0, off_down = 0, slot_stride = 0;
    uint8_t* pool = nullptr;           // n_slots * slot_stride
    float* w_router = nullptr;         // [E][H]
    float* w_router_t = nullptr;       // [H][E]
    float* w_norm = nullptr;           // [H]
    bool router_set = false;
    uint8_t* shared = nullptr;         // gate | up | down, plane layout
    int64_t sh_off_up = 0, sh_off_down = 0;
    float* sh_gate_inp = nullptr;      // [H]
    bool shared_set = false;
};

}  // namespace

struct hoard_moe_ctx {
    hoard_moe_desc desc{};
    Dims dims{};
    std::vector<LayerStore> layers;
    Scratch sc{};
    std::vector<void*> allocations;
    uint8_t* staging = nullptr;
    int64_t staging_bytes = 0;
    cudaEvent_t staging_free = nullptr;
    int64_t launches = 0;
    int decode_impl = 1;
    int gemm_min_tokens = 96;          // T at or above which the tensor-core expert path runs (0 = never)
    int routed_layer = -1;
    int routed_T = 0;
    LayerWeights* lw_dev = nullptr;    // device copy of every layer's LayerWeights (persistent kernel)
    bool decode_ok = false;            // the persistent decode kernel supports these shapes / types
    void* noalloc_scratch = nullptr;   // device address of the no-allocation decode's static array
    unsigned long long* trace = nullptr;
    int64_t trace_cap = 0;
    // residency: per-layer LRU slot pool over a host RAM tier (hoard_moe_ram_tier / hoard_moe_ensure)
    struct Residency {
        bool init = false;
        std::vector<std::array<const void*, 3>> host;   // [layer*E + expert] gate, up, down host bytes
        std::vector<std::array<const void*, 3>> direct; // the same bytes' device-accessible addresses
                                                        // (pinned host or device memory), or null
        std::vector<int> slot_of_expert;                // [layer*E + expert] -> slot or -1
        std::vector<int> expert_of_slot;                // [layer*S + slot] -> expert or -1
        std::vector<uint64_t> last_use;                 // [layer*S + slot] LRU clock
        std::vector<cudaEvent_t> ready;                 // [layer*S + slot] upload of the slot's expert done
        std::vector<char> pending;                      // [layer*S + slot] ready not yet seen complete
        std::vector<cudaEvent_t> used;                  // [layer] last hoard_moe_experts of the layer done
        std::vector<char> used_valid;
        cudaStream_t upload = nullptr;
        uint64_t clock = 0;
        int64_t hits = 0, misses = 0, bytes = 0;
    } res;
    // expert-parallel receive side (hoard_moe_ep_reserve): dispatch + h scratch for up to ep_rows rows
    int64_t ep_rows = 0;
    Scratch ep{};
    int* ep_cursor = nullptr;          // [64] pack cursors
    // expert parallelism over peer memory (hoard_moe_p2p_*)
    struct P2P {
        bool init = false, connected = false;
        int G = 0, rank = 0, epr = 0, slot_base = 0, cap = 0;
        P2PLayout L{};
        uint8_t* block = nullptr;              // this rank's symmetric block
        std::vector<uint8_t*> bases;           // every rank's block base in this process
        std::vector<void*> opened;             // IPC mappings to close
        uint8_t** peer_dev = nullptr;          // device copy of bases
        uint32_t epoch = 0;                    // barrier epochs signalled so far
        int cap_rows = 0;                      // token rows per region (max_tokens)
        int* slots = nullptr;                  // [G*cap] slot of each received entry
        int* arow = nullptr;                   // [G*cap] activation row of each received entry
        int* pos = nullptr;                    // [cap] send position of each (token, j) entry
        int* rowinfo = nullptr;                // [cap] row of the entry's token in its destination, or -1
        int* rcursor = nullptr;                // [64] rows sent per destination
        int* counts = nullptr;                 // [64] send counts per destination
        int* cursor = nullptr;                 // [64]
        int* start = nullptr;                  // [64] send offsets per destination
        Scratch rx{};                          // receive-side dispatch + h scratch for G*cap rows
        int phase = 0;                         // 0 idle, 1 sent, 2 computed
        int layer = -1, T = 0;
        const float* w = nullptr;
        unsigned long long timeout_ns = 5000000000ull;
    } p2p;
    std::string err;
};

namespace {

int fail(hoard_moe_ctx* c, int code, const std::string& msg) {
    if (c) c->err = msg;
    return code;
}

int cuda_fail(hoard_moe_ctx* c, cudaError_t e, const char* what) {
    std::string m = std::string(what) + ": " + cudaGetErrorString(e);
    return fail(c, HOARD_ECUDA, m);
}

#define HCHECK(ctx, call)                                                    \
    do {                                                                     \
        cudaError_t _e = (call);                                             \
        if (_e != cudaSuccess) return cuda_fail((ctx), _e, #call);           \
    } while (0)

template <typename T>
int dalloc(hoard_moe_ctx* c, T** p, int64_t bytes) {
    void* v = nullptr;
    if (bytes <= 0) bytes = kAlign;
    cudaError_t e = cudaMalloc(&v, (size_t)bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(c, HOARD_ENOMEM, std::string("cudaMalloc failed: ") + cudaGetErrorString(e));
    }
    c->allocations.push_back(v);
    *p = reinterpret_cast<T*>(v);
    return HOARD_OK;
}

LayerWeights layer_weights(const hoard_moe_ctx* c, int layer) {
    const LayerStore& L = c->layers[layer];
    LayerWeights lw{};
    lw.pool = L.pool;
    lw.slot_stride = L.slot_stride;
    lw.off_up = L.off_up;
    lw.off_down = L.off_down;
    lw.n_slots = c->desc.n_slots;
    lw.gate_type = L.gt;
    lw.up_type = L.ut;
    lw.down_type = L.dt;
    if (c->desc.n_ff_shexp > 0) {   // compute paths run only after check_ready saw it uploaded
        lw.shared = L.shared;
        lw.sh_off_up = L.sh_off_up;
        lw.sh_off_down = L.sh_off_down;
        lw.sh_gate_type = c->desc.shexp_gate_type;
        lw.sh_up_type = c->desc.shexp_up_type;
        lw.sh_down_type = c->desc.shexp_down_type;
        lw.sh_gate_inp = L.sh_gate_inp;
    }
    lw.w_router = L.w_router;
    lw.w_router_t = L.w_router_t;
    lw.w_norm = L.w_norm;
    return lw;
}

int check_layer(hoard_moe_ctx* c, int layer) {
    if (!c) return HOARD_EINVAL;
    if (layer < 0 || layer >= c->desc.n_layer) return fail(c, HOARD_EINVAL, "layer out of range");
    return HOARD_OK;
}

// expert positions of a token in the persistent decode kernel: the routed experts, plus the shared one
int decode_kk(const hoard_moe_ctx* c) { return c->dims.k + (c->desc.n_ff_shexp > 0 ? 1 : 0); }

int check_ready(hoard_moe_ctx* c, int layer) {
    const LayerStore& L = c->layers[layer];
    if (!L.router_set) return fail(c, HOARD_ESTATE, "router weights of this layer were never set");
    if (c->desc.n_ff_shexp > 0 && !L.shared_set) return fail(c, HOARD_ESTATE, "shared expert of this layer was never set");
    return HOARD_OK;
}

}  // namespace

extern "C" {

const char* hoard_strerror(int status) {
    switch (status) {
        case HOARD_OK: return "ok";
        case HOARD_EINVAL: return "invalid argument";
        case HOARD_ENOMEM: return "out of memory";
        case HOARD_ECUDA: return "CUDA error";
        case HOARD_ETIMEOUT: return "device wait timed out";
        case HOARD_ENCCL: return "collective failed";
        case HOARD_ESTATE: return "call out of order";
        default: return "unknown status";
    }
}

const char* hoard_moe_last_error(const hoard_moe_ctx* ctx) { return ctx ? ctx->err.c_str() : "null context"; }

int64_t hoard_moe_launch_count(const hoard_moe_ctx* ctx) { return ctx ? ctx->launches : -1; }

int hoard_moe_create(const hoard_moe_desc* d, hoard_moe_ctx** out) {
    if (!d || !out) return HOARD_EINVAL;
    *out = nullptr;
    const int H = d->n_embd, E = d->n_expert, k = d->n_expert_used, I = d->n_ff;
    if (H <= 0 || H % 256 || I <= 0 || I % 256 || E <= 0 || E > 1024 || k <= 0 || k > 16 || k > E ||
        d->n_layer <= 0 || d->n_slots <= 0 || d->n_slots > 4096 || d->max_tokens <= 0 ||
        (d->resid_type != HOARD_TYPE_F32 && d->resid_type != HOARD_TYPE_BF16))
        return HOARD_EINVAL;
    if (d->n_ff_shexp != 0 && (d->n_ff_shexp != I || !is_quant(d->shexp_gate_type) || !is_quant(d->shexp_up_type) ||
                               !is_quant(d->shexp_down_type)))
        return HOARD_EINVAL;
    for (int l = 0; l < d->n_layer; ++l) {
        if ((d->gate_types && !is_quant(d->gate_types[l])) || (d->up_types && !is_quant(d->up_types[l])) ||
            (d->down_types && !is_quant(d->down_types[l])))
            return HOARD_EINVAL;
    }
    auto* c = new hoard_moe_ctx();
    c->desc = *d;
    c->desc.gate_types = c->desc.up_types = c->desc.down_types = nullptr;  // caller's arrays are not retained
    c->dims = Dims{H, E, k, I, d->norm_topk ? 1 : 0, d->eps, d->resid_type == HOARD_TYPE_BF16 ? 1 : 0, 0};
    int rc = HOARD_OK;
    cudaError_t e = cudaSetDevice(d->device);
    if (e != cudaSuccess) {
        rc = cuda_fail(c, e, "cudaSetDevice");
        delete c;
        return rc;
    }
    c->layers.resize(d->n_layer);
    int64_t max_raw = 0;
    for (int l = 0; l < d->n_layer && rc == HOARD_OK; ++l) {
        LayerStore& L = c->layers[l];
        L.gt = d->gate_types ? d->gate_types[l] : HOARD_TYPE_Q4_K;
        L.ut = d->up_types ? d->up_types[l] : HOARD_TYPE_Q4_K;
        L.dt = d->down_types ? d->down_types[l] : HOARD_TYPE_Q6_K;
        L.gate_bytes = fmt_mat_bytes(L.gt, I, H);
        L.up_bytes = fmt_mat_bytes(L.ut, I, H);
        L.down_bytes = fmt_mat_bytes(L.dt, H, I);
        L.off_up = align_up(L.gate_bytes);
        L.off_down = L.off_up + align_up(L.up_bytes);
        L.slot_stride = L.off_down + align_up(L.down_bytes);
        max_raw = std::max(max_raw, L.gate_bytes + L.up_bytes + L.down_bytes);
        rc = dalloc(c, &L.pool, (int64_t)d->n_slots * L.slot_stride);
        if (rc == HOARD_OK) rc = dalloc(c, &L.w_router, (int64_t)E * H * 4);
        if (rc == HOARD_OK) rc = dalloc(c, &L.w_router_t, (int64_t)E * H * 4);
        if (rc == HOARD_OK) rc = dalloc(c, &L.w_norm, (int64_t)H * 4);
        if (rc == HOARD_OK && d->n_ff_shexp > 0) {
            const int64_t g = fmt_mat_bytes(d->shexp_gate_type, I, H), u = fmt_mat_bytes(d->shexp_up_type, I, H),
                          dn = fmt_mat_bytes(d->shexp_down_type, H, I);
            L.sh_off_up = align_up(g);
            L.sh_off_down = L.sh_off_up + align_up(u);
            rc = dalloc(c, &L.shared, L.sh_off_down + align_up(dn));
            if (rc == HOARD_OK) rc = dalloc(c, &L.sh_gate_inp, (int64_t)H * 4);
            max_raw = std::max(max_raw, g + u + dn);
        }
    }
    // scratch
    const int64_t T = d->max_tokens, KK = k + 1;
    Scratch& s = c->sc;
    if (rc == HOARD_OK) rc = dalloc(c, &s.fx, T * H * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &s.fx_q, T * H);
    if (rc == HOARD_OK) rc = dalloc(c, &s.fx_d, T * (H / 256) * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &s.fx_bs, T * (H / 16) * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &s.sh_gate, T * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &s.sel, T * k * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &s.w, T * k * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &s.counts, (int64_t)(d->n_slots + 2) * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &s.offsets, (int64_t)(d->n_slots + 2) * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &s.perm, T * KK * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &s.h, T * KK * I * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &s.h_q, T * KK * I);
    if (rc == HOARD_OK) rc = dalloc(c, &s.h_d, T * KK * (I / 256) * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &s.h_bs, T * KK * (I / 16) * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &s.y, T * KK * H * 4);
    const int64_t amax_rows = std::max<int64_t>(T, 2) * KK;   // >= 2 layer buffers of k rows
    if (rc == HOARD_OK) rc = dalloc(c, &s.amax, amax_rows * (I / 256) * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &s.partials, (int64_t)4096 * 1024 * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &s.sync, 4096 * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &s.xq16, T * H * 2);
    if (rc == HOARD_OK) rc = dalloc(c, &s.hq16, T * KK * I * 2);
    if (rc == HOARD_OK) rc = dalloc(c, &s.items, tc_max_items((int)T, (int)KK, d->n_slots) * (int64_t)sizeof(int2));
    if (rc == HOARD_OK) rc = dalloc(c, &s.n_items, 4);
    if (rc == HOARD_OK) rc = dalloc(c, &s.rpart, router_partial_elems((int)T, E) * 8);
    if (rc == HOARD_OK) rc = dalloc(c, &s.dcount, (int64_t)(d->n_slots + 2) * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &s.dcursor, (int64_t)(d->n_slots + 2) * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &c->staging, max_raw);
    c->staging_bytes = max_raw;
    if (rc == HOARD_OK) {
        e = cudaMemset(s.sync, 0, 4096 * 4);
        if (e == cudaSuccess) e = cudaMemset(s.amax, 0, amax_rows * (I / 256) * 4);
        if (e == cudaSuccess) e = cudaMemset(s.dcount, 0, (size_t)(d->n_slots + 2) * 4);
        if (e == cudaSuccess) e = cudaMemset(s.partials, 0, (size_t)4096 * 1024 * 4);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->staging_free, cudaEventDisableTiming);
        if (e != cudaSuccess) rc = cuda_fail(c, e, "context init");
    }
    if (rc == HOARD_OK) {
        std::vector<LayerWeights> tab(d->n_layer);
        for (int l = 0; l < d->n_layer; ++l) tab[l] = layer_weights(c, l);
        rc = dalloc(c, &c->lw_dev, (int64_t)d->n_layer * (int64_t)sizeof(LayerWeights));
        if (rc == HOARD_OK) {
            e = cudaMemcpy(c->lw_dev, tab.data(), tab.size() * sizeof(LayerWeights), cudaMemcpyHostToDevice);
            if (e != cudaSuccess) rc = cuda_fail(c, e, "layer table upload");
        }
        if (rc == HOARD_OK) {
            c->decode_ok = decode_supported(c->dims, tab.data(), d->n_layer);
            // resolved now, so that the module holding the array is loaded before the caller hands the
            // rest of the device memory to its own arena
            if (c->decode_ok && decode_static_address(&c->noalloc_scratch) != cudaSuccess) {
                cudaGetLastError();
                c->noalloc_scratch = nullptr;
            }
        }
    }
    if (rc != HOARD_OK) {
        hoard_moe_destroy(c);
        return rc;
    }
    *out = c;
    return HOARD_OK;
}

int hoard_moe_destroy(hoard_moe_ctx* c) {
    if (!c) return HOARD_EINVAL;
    cudaSetDevice(c->desc.device);
    cudaDeviceSynchronize();
    for (void* p : c->p2p.opened) cudaIpcCloseMemHandle(p);
    for (void* p : c->allocations) cudaFree(p);
    if (c->staging_free) cudaEventDestroy(c->staging_free);
    for (cudaEvent_t ev : c->res.ready) if (ev) cudaEventDestroy(ev);
    for (cudaEvent_t ev : c->res.used) if (ev) cudaEventDestroy(ev);
    if (c->res.upload) cudaStreamDestroy(c->res.upload);
    delete c;
    return HOARD_OK;
}

int64_t hoard_moe_expert_bytes(const hoard_moe_ctx* c, int layer) {
    if (!c || layer < 0 || layer >= c->desc.n_layer) return -1;
    const LayerStore& L = c->layers[layer];
    return L.gate_bytes + L.up_bytes + L.down_bytes;
}

int hoard_moe_set_router(hoard_moe_ctx* c, int layer, const float* w_router, const float* w_norm) {
    int rc = check_layer(c, layer);
    if (rc) return rc;
    if (!w_router || !w_norm) return fail(c, HOARD_EINVAL, "null router pointer");
    HCHECK(c, cudaSetDevice(c->desc.device));
    LayerStore& L = c->layers[layer];
    HCHECK(c, cudaMemcpy(L.w_router, w_router, (size_t)c->dims.E * c->dims.H * 4, cudaMemcpyDefault));
    HCHECK(c, cudaMemcpy(L.w_norm, w_norm, (size_t)c->dims.H * 4, cudaMemcpyDefault));
    HCHECK(c, launch_transpose(L.w_router, L.w_router_t, c->dims.E, c->dims.H, 0));
    HCHECK(c, cudaDeviceSynchronize());
    L.router_set = true;
    return HOARD_OK;
}

static int upload3(hoard_moe_ctx* c, uint8_t* dst_base, const int types[3], const int64_t offs[3],
                   const int64_t bytes[3], const int64_t rows[3], const void* const src[3], cudaStream_t s) {
    HCHECK(c, cudaStreamWaitEvent(s, c->staging_free, 0));
    int64_t so = 0;
    for (int m = 0; m < 3; ++m) {
        HCHECK(c, cudaMemcpyAsync(c->staging + so, src[m], (size_t)bytes[m], cudaMemcpyDefault, s));
        const int64_t nblk = bytes[m] / fmt_block_bytes(types[m]);
        (void)rows;
        HCHECK(c, launch_repack(types[m], c->staging + so, dst_base + offs[m], nblk, s));
        ++c->launches;
        so += bytes[m];
    }
    HCHECK(c, cudaEventRecord(c->staging_free, s));
    return HOARD_OK;
}

int hoard_moe_upload_expert(hoard_moe_ctx* c, int layer, int slot, const void* gate, const void* up,
                            const void* down, hoard_stream stream) {
    int rc = check_layer(c, layer);
    if (rc) return rc;
    if (slot < 0 || slot >= c->desc.n_slots) return fail(c, HOARD_EINVAL, "slot out of range");
    if (!gate || !up || !down) return fail(c, HOARD_EINVAL, "null expert pointer");
    HCHECK(c, cudaSetDevice(c->desc.device));
    LayerStore& L = c->layers[layer];
    const int types[3] = {L.gt, L.ut, L.dt};
    const int64_t offs[3] = {0, L.off_up, L.off_down};
    const int64_t bytes[3] = {L.gate_bytes, L.up_bytes, L.down_bytes};
    const int64_t rows[3] = {c->dims.I, c->dims.I, c->dims.H};
    const void* const src[3] = {gate, up, down};
    return upload3(c, L.pool + (int64_t)slot * L.slot_stride, types, offs, bytes, rows, src, (cudaStream_t)stream);
}

int hoard_moe_set_shared(hoard_moe_ctx* c, int layer, const void* gate, const void* up, const void* down,
                         const float* gate_inp) {
    int rc = check_layer(c, layer);
    if (rc) return rc;
    if (c->desc.n_ff_shexp <= 0) return fail(c, HOARD_EINVAL, "context has no shared expert");
    if (!gate || !up || !down || !gate_inp) return fail(c, HOARD_EINVAL, "null shared-expert pointer");
    HCHECK(c, cudaSetDevice(c->desc.device));
    LayerStore& L = c->layers[layer];
    const int H = c->dims.H, I = c->dims.I;
    const int types[3] = {c->desc.shexp_gate_type, c->desc.shexp_up_type, c->desc.shexp_down_type};
    const int64_t offs[3] = {0, L.sh_off_up, L.sh_off_down};
    const int64_t bytes[3] = {fmt_mat_bytes(types[0], I, H), fmt_mat_bytes(types[1], I, H), fmt_mat_bytes(types[2], H, I)};
    const int64_t rows[3] = {I, I, H};
    const void* const src[3] = {gate, up, down};
    rc = upload3(c, L.shared, types, offs, bytes, rows, src, (cudaStream_t)0);
    if (rc) return rc;
    HCHECK(c, cudaMemcpy(L.sh_gate_inp, gate_inp, (size_t)H * 4, cudaMemcpyDefault));
    HCHECK(c, cudaDeviceSynchronize());
    L.shared_set = true;
    return HOARD_OK;
}

int hoard_moe_route(hoard_moe_ctx* c, int layer, const void* x, int T, int32_t* sel, float* w,
                    hoard_stream stream) {
    int rc = check_layer(c, layer);
    if (rc) return rc;
    if (T <= 0 || T > c->desc.max_tokens) return fail(c, HOARD_EINVAL, "T out of range (1..max_tokens)");
    if (!x || !sel || !w) return fail(c, HOARD_EINVAL, "null pointer");
    if ((rc = check_ready(c, layer))) return rc;
    const LayerWeights lw = layer_weights(c, layer);
    int nl = 0;
    HCHECK(c, launch_route(c->dims, lw, x, T, c->sc.fx, sel, w, c->sc.rpart, (cudaStream_t)stream, &nl, c->sc.sync));
    c->launches += nl;
    c->routed_layer = layer;
    c->routed_T = T;
    return HOARD_OK;
}

int hoard_moe_experts(hoard_moe_ctx* c, int layer, const float* fx, const int32_t* sel, const int32_t* slot_of_sel,
                      const float* w, void* x_inout, int T, hoard_stream stream) {
    int rc = check_layer(c, layer);
    if (rc) return rc;
    if (T <= 0 || T > c->desc.max_tokens) return fail(c, HOARD_EINVAL, "T out of range (1..max_tokens)");
    if (!sel || !w || !x_inout) return fail(c, HOARD_EINVAL, "null pointer");
    if ((rc = check_ready(c, layer))) return rc;
    if (!fx) {
        if (c->routed_T < T || c->routed_layer < 0) return fail(c, HOARD_ESTATE, "no routed activations for this T");
        fx = c->sc.fx;
    }
    if (!slot_of_sel && c->desc.n_slots < c->dims.E)
        return fail(c, HOARD_EINVAL, "slot_of_sel is required when n_slots < n_expert");
    const LayerWeights lw = layer_weights(c, layer);
    int nl = 0;
    const int32_t* slots = slot_of_sel ? slot_of_sel : sel;
    if (c->gemm_min_tokens > 0 && T >= c->gemm_min_tokens && tc_supported(c->dims, lw))
        HCHECK(c, launch_experts_tc(c->dims, lw, c->sc, fx, slots, w, x_inout, T, (cudaStream_t)stream, &nl,
                                    c->trace && c->trace_cap >= tc_trace_elems() ? c->trace : nullptr));
    else
        HCHECK(c, launch_experts_grouped(c->dims, lw, c->sc, fx, slots, w, x_inout, T, true, (cudaStream_t)stream,
                                         &nl));
    c->launches += nl;
    if (c->res.init) {            // the residency layer must not overwrite these slots before this call ran
        HCHECK(c, cudaEventRecord(c->res.used[layer], (cudaStream_t)stream));
        c->res.used_valid[layer] = 1;
    }
    return HOARD_OK;
}

static int res_init(hoard_moe_ctx* c) {
    auto& r = c->res;
    if (r.init) return HOARD_OK;
    const int L = c->desc.n_layer, E = c->dims.E, S = c->desc.n_slots;
    r.host.assign((size_t)L * E, {nullptr, nullptr, nullptr});
    r.direct.assign((size_t)L * E, {nullptr, nullptr, nullptr});
    r.slot_of_expert.assign((size_t)L * E, -1);
    r.expert_of_slot.assign((size_t)L * S, -1);
    r.last_use.assign((size_t)L * S, 0);
    r.pending.assign((size_t)L * S, 0);
    r.ready.assign((size_t)L * S, nullptr);
    r.used.assign((size_t)L, nullptr);
    r.used_valid.assign((size_t)L, 0);
    HCHECK(c, cudaSetDevice(c->desc.device));
    for (auto& ev : r.ready) HCHECK(c, cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    for (auto& ev : r.used) HCHECK(c, cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    HCHECK(c, cudaStreamCreateWithFlags(&r.upload, cudaStreamNonBlocking));
    r.init = true;
    return HOARD_OK;
}

int hoard_moe_ram_tier(hoard_moe_ctx* c, int layer, int expert, const void* gate, const void* up, const void* down) {
    int rc = check_layer(c, layer);
    if (rc) return rc;
    if (expert < 0 || expert >= c->dims.E) return fail(c, HOARD_EINVAL, "expert out of range");
    if (!gate || !up || !down) return fail(c, HOARD_EINVAL, "null expert pointer");
    if ((rc = res_init(c))) return rc;
    const size_t i = (size_t)layer * c->dims.E + expert;
    c->res.host[i] = {gate, up, down};
    // pinned host (or device) bytes are read in place by the re-lay kernel: no staging copy
    std::array<const void*, 3> dir{};
    const void* src[3] = {gate, up, down};
    bool ok = true;
    for (int m = 0; m < 3 && ok; ++m) {
        cudaPointerAttributes at{};
        if (cudaPointerGetAttributes(&at, src[m]) != cudaSuccess) {
            cudaGetLastError();
            ok = false;
        } else if ((at.type == cudaMemoryTypeHost || at.type == cudaMemoryTypeDevice) && at.devicePointer &&
                   (at.type == cudaMemoryTypeHost || at.device == c->desc.device) &&
                   (reinterpret_cast<uintptr_t>(at.devicePointer) & 15) == 0) {
            dir[m] = at.devicePointer;
        } else {
            ok = false;
        }
    }
    c->res.direct[i] = ok ? dir : std::array<const void*, 3>{};
    return HOARD_OK;
}

int hoard_moe_ensure(hoard_moe_ctx* c, int layer, const int32_t* sel, int n, int32_t* slot_of_sel,
                     hoard_stream stream) {
    int rc = check_layer(c, layer);
    if (rc) return rc;
    if (!sel || !slot_of_sel || n <= 0) return fail(c, HOARD_EINVAL, "null pointer or n <= 0");
    if ((rc = res_init(c))) return rc;
    auto& r = c->res;
    const int E = c->dims.E, S = c->desc.n_slots;
    LayerStore& Ls = c->layers[layer];
    int* slot_of = &r.slot_of_expert[(size_t)layer * E];
    int* expert_of = &r.expert_of_slot[(size_t)layer * S];
    uint64_t* last = &r.last_use[(size_t)layer * S];
    for (int i = 0; i < n; ++i)
        if (sel[i] < 0 || sel[i] >= E) return fail(c, HOARD_EINVAL, "expert id out of range");
    // this call's slots are protected from eviction: stamp every hit first
    const uint64_t stamp = ++r.clock;
    for (int i = 0; i < n; ++i) {
        const int s = slot_of[sel[i]];
        if (s >= 0) last[s] = stamp;
    }
    HCHECK(c, cudaSetDevice(c->desc.device));
    std::vector<RepackJob> jobs;          // direct re-lays, one launch for all of this call's misses
    std::vector<size_t> filled;           // slots (layer * S + slot) filled by this call
    auto flush_jobs = [&]() -> int {
        if (jobs.empty()) return HOARD_OK;
        HCHECK(c, launch_repack_batch(jobs.data(), (int)jobs.size(), r.upload));
        ++c->launches;
        jobs.clear();
        return HOARD_OK;
    };
    for (int i = 0; i < n; ++i) {
        const int e = sel[i];
        int s = slot_of[e];
        if (s >= 0) {
            ++r.hits;
        } else {
            // miss: the least recently used slot that this call does not use (empty slots first)
            int victim = -1;
            for (int t = 0; t < S; ++t) {
                if (last[t] == stamp) continue;
                if (victim < 0 || (expert_of[t] < 0 && expert_of[victim] >= 0) ||
                    ((expert_of[t] < 0) == (expert_of[victim] < 0) && last[t] < last[victim]))
                    victim = t;
            }
            if (victim < 0) return fail(c, HOARD_EINVAL, "one call selects more experts than n_slots");
            const auto& h = r.host[(size_t)layer * E + e];
            if (!h[0]) return fail(c, HOARD_ESTATE, "selected expert is not in the RAM tier");
            if (expert_of[victim] >= 0) slot_of[expert_of[victim]] = -1;
            // the previous compute call of this layer may still read the victim slot
            if (r.used_valid[layer]) HCHECK(c, cudaStreamWaitEvent(r.upload, r.used[layer], 0));
            const int types[3] = {Ls.gt, Ls.ut, Ls.dt};
            const int64_t offs[3] = {0, Ls.off_up, Ls.off_down};
            const int64_t bytes[3] = {Ls.gate_bytes, Ls.up_bytes, Ls.down_bytes};
            const int64_t rows[3] = {c->dims.I, c->dims.I, c->dims.H};
            const auto& dv = r.direct[(size_t)layer * E + e];
            uint8_t* slot_base = Ls.pool + (int64_t)victim * Ls.slot_stride;
            if (dv[0]) {                      // re-laid straight from the RAM tier (over PCIe for host bytes)
                for (int m = 0; m < 3; ++m) {
                    jobs.push_back({types[m], static_cast<const uint8_t*>(dv[m]), slot_base + offs[m],
                                    bytes[m] / fmt_block_bytes(types[m])});
                    if ((int)jobs.size() == REPACK_MAX_JOBS && (rc = flush_jobs())) return rc;
                }
            } else {
                const void* const src[3] = {h[0], h[1], h[2]};
                if ((rc = upload3(c, slot_base, types, offs, bytes, rows, src, r.upload))) return rc;
            }
            filled.push_back((size_t)layer * S + victim);
            expert_of[victim] = e;
            slot_of[e] = victim;
            s = victim;
            ++r.misses;
            r.bytes += Ls.gate_bytes + Ls.up_bytes + Ls.down_bytes;
        }
        last[s] = stamp;
        slot_of_sel[i] = s;
    }
    if ((rc = flush_jobs())) return rc;
    for (size_t ri : filled) {
        HCHECK(c, cudaEventRecord(r.ready[ri], r.upload));
        r.pending[ri] = 1;
    }
    // the compute stream waits only for uploads of the slots this call uses that may still be running
    for (int i = 0; i < n; ++i) {
        const size_t ri = (size_t)layer * S + slot_of_sel[i];
        if (!r.pending[ri]) continue;
        const cudaError_t q = cudaEventQuery(r.ready[ri]);
        if (q == cudaSuccess) {
            r.pending[ri] = 0;
        } else if (q == cudaErrorNotReady) {
            HCHECK(c, cudaStreamWaitEvent((cudaStream_t)stream, r.ready[ri], 0));
        } else {
            return cuda_fail(c, q, "upload event");
        }
    }
    return HOARD_OK;
}

int hoard_moe_residency_stats(const hoard_moe_ctx* c, int64_t* hits, int64_t* misses, int64_t* bytes_uploaded) {
    if (!c || !hits || !misses || !bytes_uploaded) return HOARD_EINVAL;
    *hits = c->res.hits;
    *misses = c->res.misses;
    *bytes_uploaded = c->res.bytes;
    return HOARD_OK;
}

int hoard_moe_layers(hoard_moe_ctx* c, int layer0, int n_layers, void* x_inout, int T, int32_t* sel_out,
                     float* w_out, hoard_stream stream) {
    if (!c) return HOARD_EINVAL;
    if (n_layers <= 0 || layer0 < 0 || layer0 + n_layers > c->desc.n_layer)
        return fail(c, HOARD_EINVAL, "layer range out of bounds");
    if (T <= 0 || T > c->desc.max_tokens) return fail(c, HOARD_EINVAL, "T out of range (1..max_tokens)");
    if (!x_inout) return fail(c, HOARD_EINVAL, "null x");
    if (c->desc.n_slots < c->dims.E) return fail(c, HOARD_EINVAL, "fused layer needs every expert resident");
    for (int l = layer0; l < layer0 + n_layers; ++l) {
        int rc = check_ready(c, l);
        if (rc) return rc;
    }
    const int k = c->dims.k;
    HCHECK(c, cudaSetDevice(c->desc.device));
    if (T == 1 && c->decode_impl == 1 && c->decode_ok) {
        unsigned long long* tr = nullptr;
        if (c->trace && (int64_t)decode_grid() * n_layers * decode_trace_phases() <= c->trace_cap) tr = c->trace;
        HCHECK(c, launch_decode_persistent(c->dims, decode_kk(c), c->desc.shexp_down_type, c->lw_dev + layer0, n_layers,
                                           c->sc, x_inout, T, sel_out, w_out, (cudaStream_t)stream, tr));
        ++c->launches;
        return HOARD_OK;
    }
    for (int l = layer0; l < layer0 + n_layers; ++l) {
        const int64_t o = (int64_t)(l - layer0) * T * k;
        int32_t* sel = sel_out ? sel_out + o : c->sc.sel;
        float* w = w_out ? w_out + o : c->sc.w;
        const LayerWeights lw = layer_weights(c, l);
        const bool gemm = c->gemm_min_tokens > 0 && T >= c->gemm_min_tokens && tc_supported(c->dims, lw);
        if (!gemm && route_fused_supported(c->dims, T) && gateup_sw_supported(c->dims, lw) &&
            down_sw_supported(c->dims, lw)) {
            // small batches: graph A's tail, the Q8_K of fx and the dispatch in one kernel, then the
            // streaming expert kernels
            const int KK = k + (lw.shared ? 1 : 0);
            unsigned long long* st = c->trace && c->trace_cap >= 6 ? c->trace : nullptr;
            HCHECK(c, launch_route_fused(c->dims, lw, c->sc, x_inout, T, KK, sel, w, 1 << 20, (cudaStream_t)stream, st));
            int nl = 1;
            HCHECK(c, launch_experts_grouped(c->dims, lw, c->sc, c->sc.fx, sel, w, x_inout, T, true,
                                             (cudaStream_t)stream, &nl, true, st ? st + 2 : nullptr));
            c->launches += nl;
            c->routed_layer = l;
            c->routed_T = T;
            if (c->res.init) {
                HCHECK(c, cudaEventRecord(c->res.used[l], (cudaStream_t)stream));
                c->res.used_valid[l] = 1;
            }
            continue;
        }
        int rc = hoard_moe_route(c, l, x_inout, T, sel, w, stream);
        if (rc) return rc;
        rc = hoard_moe_experts(c, l, nullptr, sel, nullptr, w, x_inout, T, stream);
        if (rc) return rc;
    }
    return HOARD_OK;
}

int hoard_moe_layer(hoard_moe_ctx* c, int layer, void* x_inout, int T, int32_t* sel_out, float* w_out,
                    hoard_stream stream) {
    return hoard_moe_layers(c, layer, 1, x_inout, T, sel_out, w_out, stream);
}

int hoard_moe_decode_noalloc(hoard_moe_ctx* c, int layer0, int n_layers, void* x_inout, int32_t* sel_out,
                             float* w_out, hoard_stream stream) {
    if (!c) return HOARD_EINVAL;
    if (n_layers <= 0 || layer0 < 0 || layer0 + n_layers > c->desc.n_layer)
        return fail(c, HOARD_EINVAL, "layer range out of bounds");
    if (!x_inout) return fail(c, HOARD_EINVAL, "null x");
    if ((sel_out == nullptr) != (w_out == nullptr)) return fail(c, HOARD_EINVAL, "sel_out and w_out go together");
    if (!decode_static_fits(c->dims, decode_kk(c)))
        return fail(c, HOARD_EINVAL, "shape exceeds the static decode scratch (needs n_expert_used <= 16, "
                                     "n_ff <= 1024, n_expert <= 512)");
    if (!c->decode_ok || c->desc.n_slots < c->dims.E)
        return fail(c, HOARD_ESTATE, "the persistent decode kernel does not support this context");
    for (int l = layer0; l < layer0 + n_layers; ++l) {
        int rc = check_ready(c, l);
        if (rc) return rc;
    }
    HCHECK(c, cudaSetDevice(c->desc.device));
    if (!c->noalloc_scratch) return fail(c, HOARD_ESTATE, "the static decode scratch could not be resolved on this device");
    HCHECK(c, launch_decode_static(c->dims, decode_kk(c), c->desc.shexp_down_type, c->lw_dev + layer0, n_layers,
                                   c->noalloc_scratch, x_inout, sel_out, w_out, (cudaStream_t)stream));
    ++c->launches;
    return HOARD_OK;
}

int hoard_moe_set_decode_impl(hoard_moe_ctx* c, int impl) {
    if (!c || impl < 0 || impl > 1) return HOARD_EINVAL;
    c->decode_impl = impl;
    return HOARD_OK;
}

int hoard_moe_ep_reserve(hoard_moe_ctx* c, int64_t max_rows) {
    if (!c || max_rows <= 0 || max_rows > (int64_t)1 << 30) return c ? fail(c, HOARD_EINVAL, "max_rows out of range") : HOARD_EINVAL;
    if (max_rows <= c->ep_rows) return HOARD_OK;
    HCHECK(c, cudaSetDevice(c->desc.device));
    Scratch& e = c->ep;
    const int64_t NS2 = (int64_t)c->desc.n_slots + 2;
    int rc = dalloc(c, &e.counts, NS2 * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &e.offsets, NS2 * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &e.perm, max_rows * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &e.hq16, max_rows * c->dims.I * 2);
    if (rc == HOARD_OK) rc = dalloc(c, &e.items, tc_max_items((int)max_rows, 1, c->desc.n_slots) * (int64_t)sizeof(int2));
    if (rc == HOARD_OK) rc = dalloc(c, &e.n_items, 4);
    if (rc == HOARD_OK) rc = dalloc(c, &e.dcount, NS2 * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &e.dcursor, NS2 * 4);
    if (rc == HOARD_OK && !c->ep_cursor) rc = dalloc(c, &c->ep_cursor, 64 * 4);
    if (rc != HOARD_OK) return rc;
    HCHECK(c, cudaMemset(e.dcount, 0, (size_t)NS2 * 4));
    e.sync = c->sc.sync;
    c->ep_rows = max_rows;
    return HOARD_OK;
}

int hoard_moe_ep_pack(hoard_moe_ctx* c, int layer, const int32_t* sel, int T, int n_ranks, int experts_per_rank,
                      int32_t* send_counts, int32_t* pos_of_entry, int32_t* send_expert, uint16_t* send_rows,
                      hoard_stream stream) {
    int rc = check_layer(c, layer);
    if (rc) return rc;
    if (T <= 0 || T > c->desc.max_tokens) return fail(c, HOARD_EINVAL, "T out of range (1..max_tokens)");
    if (n_ranks < 1 || n_ranks > 64 || experts_per_rank < 1 || (int64_t)n_ranks * experts_per_rank < c->dims.E)
        return fail(c, HOARD_EINVAL, "n_ranks * experts_per_rank must cover n_expert (n_ranks <= 64)");
    if (!sel || !send_counts || !pos_of_entry || !send_expert || !send_rows) return fail(c, HOARD_EINVAL, "null pointer");
    if (c->routed_layer != layer || c->routed_T < T)
        return fail(c, HOARD_ESTATE, "hoard_moe_route(layer, ..., T) must run first on this stream");
    if (!c->ep_cursor && (rc = dalloc(c, &c->ep_cursor, 64 * 4))) return rc;
    HCHECK(c, cudaSetDevice(c->desc.device));
    int nl = 0;
    HCHECK(c, launch_q8_rows(c->sc.fx, T, c->dims.H, c->sc.xq16, (cudaStream_t)stream));
    ++nl;
    HCHECK(c, launch_ep_pack(sel, T, c->dims.k, n_ranks, experts_per_rank, c->sc.xq16, c->dims.H, send_counts,
                             c->ep_cursor, pos_of_entry, send_expert, send_rows, c->sc.sync, (cudaStream_t)stream, &nl));
    c->launches += nl;
    return HOARD_OK;
}

int hoard_moe_ep_experts(hoard_moe_ctx* c, int layer, const uint16_t* rows, const int32_t* slot_of_row, int R,
                         uint16_t* y_out, hoard_stream stream) {
    int rc = check_layer(c, layer);
    if (rc) return rc;
    if (R < 0 || R > c->ep_rows) return fail(c, HOARD_EINVAL, "R out of range (0..hoard_moe_ep_reserve's max_rows)");
    if (R == 0) return HOARD_OK;
    if (!rows || !slot_of_row || !y_out) return fail(c, HOARD_EINVAL, "null pointer");
    const LayerWeights lw = layer_weights(c, layer);
    if (!tc_supported(c->dims, lw)) return fail(c, HOARD_EINVAL, "expert types unsupported by the tensor-core path");
    HCHECK(c, cudaSetDevice(c->desc.device));
    int nl = 0;
    HCHECK(c, launch_experts_tc_rows(c->dims, lw, c->ep, rows, slot_of_row, R, y_out, (cudaStream_t)stream, &nl));
    c->launches += nl;
    return HOARD_OK;
}

int hoard_moe_ep_combine(hoard_moe_ctx* c, const float* w, const int32_t* pos_of_entry, const uint16_t* y_back,
                         void* x_inout, int T, hoard_stream stream) {
    if (!c) return HOARD_EINVAL;
    if (T <= 0 || T > c->desc.max_tokens) return fail(c, HOARD_EINVAL, "T out of range (1..max_tokens)");
    if (!w || !pos_of_entry || !y_back || !x_inout) return fail(c, HOARD_EINVAL, "null pointer");
    HCHECK(c, cudaSetDevice(c->desc.device));
    HCHECK(c, launch_combine_rows(c->dims, y_back, pos_of_entry, w, x_inout, T, (cudaStream_t)stream));
    ++c->launches;
    return HOARD_OK;
}

int hoard_moe_set_gemm_ctas(hoard_moe_ctx* c, int ctas) {
    if (!c || ctas < 0) return HOARD_EINVAL;
    c->dims.gemm_ctas = ctas;
    return HOARD_OK;
}

int hoard_moe_set_top_k(hoard_moe_ctx* c, int k) {
    if (!c) return HOARD_EINVAL;
    if (k < 1 || k > c->desc.n_expert_used) return fail(c, HOARD_EINVAL, "k must be 1..n_expert_used");
    c->dims.k = k;
    std::vector<LayerWeights> tab(c->desc.n_layer);
    for (int l = 0; l < c->desc.n_layer; ++l) tab[l] = layer_weights(c, l);
    HCHECK(c, cudaSetDevice(c->desc.device));
    c->decode_ok = decode_supported(c->dims, tab.data(), c->desc.n_layer);
    if (c->decode_ok && !c->noalloc_scratch && decode_static_address(&c->noalloc_scratch) != cudaSuccess) {
        cudaGetLastError();
        c->noalloc_scratch = nullptr;
    }
    return HOARD_OK;
}

int hoard_moe_set_gemm_min_tokens(hoard_moe_ctx* c, int min_tokens) {
    if (!c || min_tokens < 0) return HOARD_EINVAL;
    c->gemm_min_tokens = min_tokens;
    return HOARD_OK;
}

int hoard_moe_set_trace(hoard_moe_ctx* c, uint64_t* dev_buf, int64_t capacity) {
    if (!c || capacity < 0 || (capacity > 0 && !dev_buf)) return HOARD_EINVAL;
    c->trace = capacity > 0 ? reinterpret_cast<unsigned long long*>(dev_buf) : nullptr;
    c->trace_cap = capacity;
    return HOARD_OK;
}

int hoard_moe_trace_layout(const hoard_moe_ctx* c, int* ctas, int* phases) {
    if (!c || !ctas || !phases) return HOARD_EINVAL;
    *ctas = decode_grid();
    *phases = decode_trace_phases();
    return HOARD_OK;
}

namespace {
// waits for `stream`, reads and clears the device error word at `word`, and maps its bits to a status
int read_error_word(hoard_moe_ctx* c, unsigned* word, hoard_stream stream) {
    HCHECK(c, cudaSetDevice(c->desc.device));
    HCHECK(c, cudaStreamSynchronize((cudaStream_t)stream));
    unsigned flags = 0;
    HCHECK(c, cudaMemcpy(&flags, word, 4, cudaMemcpyDeviceToHost));
    if (flags) {
        const unsigned zero = 0;
        HCHECK(c, cudaMemcpy(word, &zero, 4, cudaMemcpyHostToDevice));
        if (flags & 2u) return fail(c, HOARD_ETIMEOUT, "a device-side wait gave up");
        if (flags & 4u) return fail(c, HOARD_EINVAL, "decode router sums left the fixed-point range");
        return fail(c, HOARD_EINVAL, "an expert or slot id was out of range (entries skipped)");
    }
    return HOARD_OK;
}
}  // namespace

int hoard_moe_sync_status(hoard_moe_ctx* c, hoard_stream stream) {
    if (!c) return HOARD_EINVAL;
    return read_error_word(c, c->sc.sync, stream);
}

int hoard_moe_decode_noalloc_status(hoard_moe_ctx* c, hoard_stream stream) {
    if (!c) return HOARD_EINVAL;
    if (!c->noalloc_scratch) return fail(c, HOARD_ESTATE, "the static decode scratch could not be resolved on this device");
    return read_error_word(c, reinterpret_cast<unsigned*>(static_cast<uint8_t*>(c->noalloc_scratch) +
                                                           decode_static_error_offset()),
                           stream);
}

// ---- expert parallelism over peer memory ----

namespace {

struct P2PHandle {
    uint32_t magic, version;
    int32_t G, rank, cap, H;
    int64_t bytes;
    cudaIpcMemHandle_t ipc;
};
static_assert(sizeof(P2PHandle) <= HOARD_P2P_HANDLE_BYTES, "handle blob too small");
constexpr uint32_t kP2PMagic = 0x50324850u;   // "PH2P"

P2PSend p2p_args(const hoard_moe_ctx* c) {
    P2PSend p{};
    p.peer = c->p2p.peer_dev;
    p.L = c->p2p.L;
    p.G = c->p2p.G;
    p.rank = c->p2p.rank;
    p.cap = c->p2p.cap;
    p.cap_rows = c->p2p.cap_rows;
    p.H = c->dims.H;
    p.epr = c->p2p.epr;
    return p;
}

int p2p_connect(hoard_moe_ctx* c) {
    HCHECK(c, cudaMemcpy(c->p2p.peer_dev, c->p2p.bases.data(), c->p2p.G * sizeof(uint8_t*), cudaMemcpyHostToDevice));
    c->p2p.connected = true;
    c->p2p.phase = 0;
    return HOARD_OK;
}

}  // namespace

int hoard_moe_p2p_init(hoard_moe_ctx* c, int n_ranks, int rank, int experts_per_rank, int slot_base) {
    if (!c) return HOARD_EINVAL;
    auto& P = c->p2p;
    if (P.init) return fail(c, HOARD_ESTATE, "peer-memory expert parallelism already initialised");
    if (n_ranks < 1 || n_ranks > 64 || rank < 0 || rank >= n_ranks || experts_per_rank < 1 ||
        (int64_t)n_ranks * experts_per_rank < c->dims.E || slot_base < 0)
        return fail(c, HOARD_EINVAL, "need 1 <= n_ranks <= 64, 0 <= rank < n_ranks, n_ranks * experts_per_rank >= n_expert");
    const int own = std::max(0, std::min(experts_per_rank, c->dims.E - rank * experts_per_rank));
    if (slot_base + own > c->desc.n_slots) return fail(c, HOARD_EINVAL, "this rank's experts do not fit the pool");
    if (c->desc.n_ff_shexp > 0) return fail(c, HOARD_EINVAL, "layers with a shared expert are not supported");
    HCHECK(c, cudaSetDevice(c->desc.device));
    const int64_t cap = (int64_t)c->desc.max_tokens * c->dims.k;
    if (cap * n_ranks > ((int64_t)1 << 30)) return fail(c, HOARD_EINVAL, "max_tokens * k * n_ranks too large");
    P.G = n_ranks;
    P.rank = rank;
    P.epr = experts_per_rank;
    P.slot_base = slot_base;
    P.cap = (int)cap;
    P.cap_rows = c->desc.max_tokens;
    P.L = p2p_layout(n_ranks, P.cap, P.cap_rows, c->dims.H);
    const int64_t R = cap * n_ranks;
    Scratch& x = P.rx;
    const int64_t NS2 = (int64_t)c->desc.n_slots + 2;
    int rc = dalloc(c, &P.block, P.L.bytes);
    if (rc == HOARD_OK) rc = dalloc(c, &P.peer_dev, 64 * sizeof(uint8_t*));
    if (rc == HOARD_OK) rc = dalloc(c, &P.slots, R * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &P.arow, R * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &P.pos, cap * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &P.rowinfo, cap * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &P.rcursor, 64 * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &P.counts, 64 * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &P.cursor, 64 * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &P.start, 64 * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &x.counts, NS2 * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &x.offsets, NS2 * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &x.perm, R * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &x.hq16, R * c->dims.I * 2);
    if (rc == HOARD_OK) rc = dalloc(c, &x.items, tc_max_items((int)R, 1, c->desc.n_slots) * (int64_t)sizeof(int2));
    if (rc == HOARD_OK) rc = dalloc(c, &x.n_items, 4);
    if (rc == HOARD_OK) rc = dalloc(c, &x.dcount, NS2 * 4);
    if (rc == HOARD_OK) rc = dalloc(c, &x.dcursor, NS2 * 4);
    if (rc != HOARD_OK) return rc;
    HCHECK(c, cudaMemset(P.block, 0, (size_t)P.L.bytes));
    HCHECK(c, cudaMemset(x.dcount, 0, (size_t)NS2 * 4));
    HCHECK(c, cudaDeviceSynchronize());
    x.sync = c->sc.sync;
    P.bases.assign(n_ranks, nullptr);
    P.bases[rank] = P.block;
    P.init = true;
    return HOARD_OK;
}

int hoard_moe_p2p_handle(hoard_moe_ctx* c, void* out) {
    if (!c || !out) return HOARD_EINVAL;
    if (!c->p2p.init) return fail(c, HOARD_ESTATE, "hoard_moe_p2p_init must run first");
    HCHECK(c, cudaSetDevice(c->desc.device));
    P2PHandle h{};
    h.magic = kP2PMagic;
    h.version = 2;
    h.G = c->p2p.G;
    h.rank = c->p2p.rank;
    h.cap = c->p2p.cap;
    h.H = c->dims.H;
    h.bytes = c->p2p.L.bytes;
    HCHECK(c, cudaIpcGetMemHandle(&h.ipc, c->p2p.block));
    std::memset(out, 0, HOARD_P2P_HANDLE_BYTES);
    std::memcpy(out, &h, sizeof(h));
    return HOARD_OK;
}

int hoard_moe_p2p_open(hoard_moe_ctx* c, const void* handles) {
    if (!c || !handles) return HOARD_EINVAL;
    auto& P = c->p2p;
    if (!P.init) return fail(c, HOARD_ESTATE, "hoard_moe_p2p_init must run first");
    if (P.connected) return fail(c, HOARD_ESTATE, "already connected (hoard_moe_p2p_close first)");
    HCHECK(c, cudaSetDevice(c->desc.device));
    for (int s = 0; s < P.G; ++s) {
        P2PHandle h;
        std::memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)s * HOARD_P2P_HANDLE_BYTES, sizeof(h));
        if (h.magic != kP2PMagic || h.version != 2 || h.G != P.G || h.rank != s || h.cap != P.cap ||
            h.H != c->dims.H || h.bytes != P.L.bytes)
            return fail(c, HOARD_EINVAL, "peer handle " + std::to_string(s) + " does not match this group");
    }
    for (int s = 0; s < P.G; ++s) {
        if (s == P.rank) continue;
        P2PHandle h;
        std::memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)s * HOARD_P2P_HANDLE_BYTES, sizeof(h));
        void* ptr = nullptr;
        HCHECK(c, cudaIpcOpenMemHandle(&ptr, h.ipc, cudaIpcMemLazyEnablePeerAccess));
        P.opened.push_back(ptr);
        P.bases[s] = static_cast<uint8_t*>(ptr);
    }
    return p2p_connect(c);
}

int hoard_moe_p2p_attach(hoard_moe_ctx* c, hoard_moe_ctx* const* peers) {
    if (!c || !peers) return HOARD_EINVAL;
    auto& P = c->p2p;
    if (!P.init) return fail(c, HOARD_ESTATE, "hoard_moe_p2p_init must run first");
    if (P.connected) return fail(c, HOARD_ESTATE, "already connected (hoard_moe_p2p_close first)");
    if (peers[P.rank] != c) return fail(c, HOARD_EINVAL, "peers[rank] must be this context");
    HCHECK(c, cudaSetDevice(c->desc.device));
    for (int s = 0; s < P.G; ++s) {
        const hoard_moe_ctx* q = peers[s];
        if (!q || !q->p2p.init || q->p2p.G != P.G || q->p2p.rank != s || q->p2p.cap != P.cap ||
            q->dims.H != c->dims.H)
            return fail(c, HOARD_EINVAL, "peer " + std::to_string(s) + " does not match this group");
        if (q->desc.device != c->desc.device) {
            cudaError_t e = cudaDeviceEnablePeerAccess(q->desc.device, 0);
            if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
            else if (e != cudaSuccess) return cuda_fail(c, e, "cudaDeviceEnablePeerAccess");
        }
        P.bases[s] = q->p2p.block;
    }
    return p2p_connect(c);
}

int hoard_moe_p2p_close(hoard_moe_ctx* c) {
    if (!c) return HOARD_EINVAL;
    auto& P = c->p2p;
    if (!P.init) return HOARD_OK;
    HCHECK(c, cudaSetDevice(c->desc.device));
    HCHECK(c, cudaDeviceSynchronize());
    for (void* p : P.opened) cudaIpcCloseMemHandle(p);
    P.opened.clear();
    for (int s = 0; s < P.G; ++s)
        if (s != P.rank) P.bases[s] = nullptr;
    HCHECK(c, cudaMemset(P.block + P.L.flags, 0, 256));
    HCHECK(c, cudaDeviceSynchronize());
    P.epoch = 0;
    P.connected = false;
    P.phase = 0;
    return HOARD_OK;
}

int hoard_moe_p2p_set_timeout(hoard_moe_ctx* c, double seconds) {
    if (!c || !(seconds > 0) || seconds > 3600) return c ? fail(c, HOARD_EINVAL, "timeout out of range") : HOARD_EINVAL;
    c->p2p.timeout_ns = (unsigned long long)(seconds * 1e9);
    return HOARD_OK;
}

int hoard_moe_p2p_send(hoard_moe_ctx* c, int layer, const void* x, int T, int32_t* sel_out, float* w_out,
                       hoard_stream stream) {
    int rc = check_layer(c, layer);
    if (rc) return rc;
    auto& P = c->p2p;
    if (!P.connected) return fail(c, HOARD_ESTATE, "peer group not connected (hoard_moe_p2p_open / attach)");
    if (P.phase != 0) return fail(c, HOARD_ESTATE, "hoard_moe_p2p_finish of the previous layer has not run");
    if (!tc_supported(c->dims, layer_weights(c, layer)))
        return fail(c, HOARD_EINVAL, "expert types unsupported by the tensor-core path");
    int32_t* sel = sel_out ? sel_out : c->sc.sel;
    float* w = w_out ? w_out : c->sc.w;
    if ((rc = hoard_moe_route(c, layer, x, T, sel, w, stream))) return rc;
    const cudaStream_t s = (cudaStream_t)stream;
    HCHECK(c, launch_q8_rows(c->sc.fx, T, c->dims.H, c->sc.xq16, s));
    int nl = 1;
    const P2PSend a = p2p_args(c);
    HCHECK(c, launch_p2p_send(a, sel, T, c->dims.k, c->sc.xq16, P.counts, P.cursor, P.start, P.rcursor, P.pos,
                              P.rowinfo, c->sc.sync, s, &nl));
    HCHECK(c, launch_p2p_signal(a, ++P.epoch, s));
    c->launches += nl + 1;
    P.phase = 1;
    P.layer = layer;
    P.T = T;
    P.w = w;
    return HOARD_OK;
}

int hoard_moe_p2p_compute(hoard_moe_ctx* c, hoard_stream stream) {
    if (!c) return HOARD_EINVAL;
    auto& P = c->p2p;
    if (P.phase != 1) return fail(c, HOARD_ESTATE, "hoard_moe_p2p_send must run first");
    HCHECK(c, cudaSetDevice(c->desc.device));
    const cudaStream_t s = (cudaStream_t)stream;
    const P2PSend a = p2p_args(c);
    HCHECK(c, launch_p2p_wait(P.block, P.L, P.G, P.epoch, P.timeout_ns, c->sc.sync, s));
    int nl = 1;
    HCHECK(c, launch_p2p_experts(c->dims, layer_weights(c, P.layer), P.rx, a, P.block, P.slot_base, P.slots, P.arow, s,
                                 &nl));
    HCHECK(c, launch_p2p_signal(a, ++P.epoch, s));
    c->launches += nl + 1;
    P.phase = 2;
    return HOARD_OK;
}

int hoard_moe_p2p_finish(hoard_moe_ctx* c, void* x_inout, hoard_stream stream) {
    if (!c) return HOARD_EINVAL;
    auto& P = c->p2p;
    if (P.phase != 2) return fail(c, HOARD_ESTATE, "hoard_moe_p2p_compute must run first");
    if (!x_inout) return fail(c, HOARD_EINVAL, "null x");
    HCHECK(c, cudaSetDevice(c->desc.device));
    const cudaStream_t s = (cudaStream_t)stream;
    HCHECK(c, launch_p2p_wait(P.block, P.L, P.G, P.epoch, P.timeout_ns, c->sc.sync, s));
    HCHECK(c, launch_combine_rows(c->dims, reinterpret_cast<const uint16_t*>(P.block + P.L.yback), P.pos, P.w,
                                  x_inout, P.T, s));
    c->launches += 2;
    P.phase = 0;
    return HOARD_OK;
}

int hoard_moe_p2p_layers(hoard_moe_ctx* c, int layer0, int n_layers, void* x_inout, int T, int32_t* sel_out,
                         float* w_out, hoard_stream stream) {
    if (!c) return HOARD_EINVAL;
    if (n_layers <= 0 || layer0 < 0 || layer0 + n_layers > c->desc.n_layer)
        return fail(c, HOARD_EINVAL, "layer range out of bounds");
    for (int l = layer0; l < layer0 + n_layers; ++l) {
        const int64_t o = (int64_t)(l - layer0) * T * c->dims.k;
        int rc = hoard_moe_p2p_send(c, l, x_inout, T, sel_out ? sel_out + o : nullptr, w_out ? w_out + o : nullptr,
                                    stream);
        if (!rc) rc = hoard_moe_p2p_compute(c, stream);
        if (!rc) rc = hoard_moe_p2p_finish(c, x_inout, stream);
        if (rc) return rc;
    }
    return HOARD_OK;
}

}  // extern "C"
