// af_engine.cu -- a whole greedy decode step in C++ on this library's kernels.
//
// Reference behaviour (AtomFlow):
//   include/core/engine.h            AtomFlowEngine: initialize, inject_token,
//                                    forward_pass, get_output_token, current_pos_
//   src/core/engine.cu:56-234        static arenas (weights, activations, KV cache)
//   src/core/engine.cu:262-521       forward_pass: embedding, 28 x {RMSNorm, QKV,
//                                    RoPE + KV write, attention, O, residual,
//                                    RMSNorm, gate, up, SwiGLU, down, residual},
//                                    final RMSNorm, lm_head, argmax
//   include/memory/weight_loader.h   the .bin file (mmap, 256-byte header, blocks
//                                    padded to 256 bytes) written by
//                                    tools/quantize_weights.py:320-427
//
// The file is mapped, validated against its header, and copied to the device
// once: its block layout is already 256-byte aligned, so every tensor is a
// pointer into one device arena at the block's file offset.  The step keeps
// the token id and the position in device ints; af_engine_capture records it
// as a CUDA graph.

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#include "../../include/atomflow_b200.h"
#include "af_internal.h"

namespace {

constexpr size_t kAlign = 256;
constexpr int kGroup = 128;
constexpr float kNormEps = 1e-5f;       // RMSNorm epsilon of the Llama 3 config
constexpr float kRopeBase = 500000.0f;  // RoPE theta of Llama 3 (helpers.cu build_rope_cache)

size_t pad(size_t n) { return (n + kAlign - 1) / kAlign * kAlign; }

struct Header {
    char magic[4];
    int version, group_size, dim, ffn, n_layers, n_heads, n_kv_heads, vocab, max_seq_len;
};

struct Linear {
    const uint8_t* w;
    const uint16_t* s;
    int N, K;
};

struct Layer {
    const float* in_norm;
    const float* post_norm;
    Linear qkv, o, gate, up, down;
    __half* k_cache;
    __half* v_cache;
};

}  // namespace

struct af_engine {
    Header h{};
    int HD = 0, QD = 0, KVD = 0, QKV = 0;
    int max_seq = 0;
    af_engine_mode mode = AF_ENGINE_EXACT;
    af_argmax_mode amode = AF_ARGMAX_REF_COMPAT;
    size_t file_bytes = 0;
    cudaStream_t stream = nullptr;
    unsigned char* arena = nullptr;     // the file's blocks
    unsigned char* acts = nullptr;      // activations, state ints, workspaces
    unsigned char* kv = nullptr;        // KV cache, [layer][k|v][max_seq][KVD]
    const float* embed = nullptr;
    const float* final_norm = nullptr;
    const uint16_t* lm_head = nullptr;
    std::vector<Layer> layers;
    float* cos_tab = nullptr;
    float* sin_tab = nullptr;
    __half *x = nullptr, *xn = nullptr, *qkv = nullptr, *attn = nullptr, *hbuf = nullptr;
    float* logits = nullptr;
    int* d_token = nullptr;
    int* d_pos = nullptr;
    void* attn_ws = nullptr;
    size_t attn_ws_bytes = 0;
    void* lm_ws = nullptr;
    size_t lm_ws_bytes = 0;
    void* chain_ws = nullptr;
    size_t chain_ws_bytes = 0;
    std::vector<std::vector<af_chain_op>> segments;   // exact mode: the chain launches of a step
    cudaGraphExec_t graph = nullptr;
    bool stepped = false;
    int launches = 0;
    // tensor parallelism (world > 1): this rank's heads, FFN rows and vocabulary rows
    af_tp_comm* comm = nullptr;
    int rank = 0, world = 1;
    int NHl = 0, NKVl = 0, FFNl = 0, v0 = 0, v1 = 0;
    std::vector<void*> owned;   // per-tensor device buffers of a sharded load
};

namespace {

// Tensor parallelism: copies this rank's part of every tensor out of the mapped
// file into its own device buffer (Megatron split; the row-split K shards hold
// whole 128-wide scale groups, so their scales are the full matrix's):
//   qkv   rows of the rank's query heads, then of its kv heads' k and v
//   o     the columns of the rank's heads (K split)
//   gate, up   rows [r F/w, (r+1) F/w)
//   down  columns [r F/w, (r+1) F/w) (K split)
//   lm_head    vocabulary rows [r V/w, (r+1) V/w)
// The embedding and the norms are replicated.
af_status load_shards(af_engine* e, const unsigned char* f, size_t embed_off, size_t fnorm_off, size_t lm_off,
                      const std::vector<size_t>& blocks) {
    const Header& h = e->h;
    const int w = e->world, r = e->rank, HD = e->HD;
    cudaError_t ce = cudaSuccess;
    // rows x width bytes, source pitch spitch, from file offset src
    auto copy2d = [&](size_t src, size_t width, size_t rows, size_t spitch) -> unsigned char* {
        unsigned char* d = nullptr;
        if (ce != cudaSuccess) return nullptr;
        ce = cudaMalloc(&d, std::max<size_t>(width * rows, 16));
        if (ce != cudaSuccess) return nullptr;
        e->owned.push_back(d);
        ce = cudaMemcpy2D(d, width, f + src, spitch, width, rows, cudaMemcpyHostToDevice);
        return d;
    };
    const size_t D = h.dim, F = h.ffn, G = D / kGroup, GF = F / kGroup;
    e->embed = reinterpret_cast<const float*>(copy2d(embed_off, (size_t)h.vocab * D * 4, 1, 0));
    e->final_norm = reinterpret_cast<const float*>(copy2d(fnorm_off, D * 4, 1, 0));
    e->lm_head = reinterpret_cast<const uint16_t*>(
        copy2d(lm_off + (size_t)e->v0 * D * 2, (size_t)(e->v1 - e->v0) * D * 2, 1, 0));
    e->layers.resize(h.n_layers);
    const int hq = e->NHl, hk = e->NKVl;
    for (int l = 0; l < h.n_layers && ce == cudaSuccess; ++l) {
        const size_t* b = &blocks[(size_t)l * 12];
        Layer& L = e->layers[l];
        L.in_norm = reinterpret_cast<const float*>(copy2d(b[0], D * 4, 1, 0));
        L.post_norm = reinterpret_cast<const float*>(copy2d(b[1], D * 4, 1, 0));
        // qkv: three row ranges packed [Q_r | K_r | V_r]
        {
            const size_t rq = (size_t)hq * HD, rk = (size_t)hk * HD;
            const size_t starts[3] = {(size_t)r * rq, (size_t)h.n_heads * HD + (size_t)r * rk,
                                      (size_t)(h.n_heads + h.n_kv_heads) * HD + (size_t)r * rk};
            const size_t counts[3] = {rq, rk, rk};
            unsigned char* wq = nullptr;
            unsigned char* sq = nullptr;
            const size_t rows = rq + 2 * rk;
            if (ce == cudaSuccess) ce = cudaMalloc(&wq, rows * D);
            if (ce == cudaSuccess) { e->owned.push_back(wq); ce = cudaMalloc(&sq, rows * G * 2); }
            if (ce == cudaSuccess) e->owned.push_back(sq);
            size_t at_row = 0;
            for (int p = 0; p < 3 && ce == cudaSuccess; ++p) {
                ce = cudaMemcpy(wq + at_row * D, f + b[2] + starts[p] * D, counts[p] * D, cudaMemcpyHostToDevice);
                if (ce == cudaSuccess)
                    ce = cudaMemcpy(sq + at_row * G * 2, f + b[3] + starts[p] * G * 2, counts[p] * G * 2,
                                    cudaMemcpyHostToDevice);
                at_row += counts[p];
            }
            L.qkv = {wq, reinterpret_cast<const uint16_t*>(sq), (int)rows, (int)D};
        }
        // o: K split by heads
        {
            const size_t kc = D / w;
            unsigned char* wo = copy2d(b[4] + (size_t)r * kc, kc, D, D);
            unsigned char* so = copy2d(b[5] + (size_t)r * (G / w) * 2, (G / w) * 2, D, G * 2);
            L.o = {wo, reinterpret_cast<const uint16_t*>(so), (int)D, (int)kc};
        }
        // gate, up: rows
        {
            const size_t rows = F / w;
            unsigned char* wg = copy2d(b[6] + (size_t)r * rows * D, rows * D, 1, 0);
            unsigned char* sg = copy2d(b[7] + (size_t)r * rows * G * 2, rows * G * 2, 1, 0);
            unsigned char* wu = copy2d(b[8] + (size_t)r * rows * D, rows * D, 1, 0);
            unsigned char* su = copy2d(b[9] + (size_t)r * rows * G * 2, rows * G * 2, 1, 0);
            L.gate = {wg, reinterpret_cast<const uint16_t*>(sg), (int)rows, (int)D};
            L.up = {wu, reinterpret_cast<const uint16_t*>(su), (int)rows, (int)D};
        }
        // down: K split
        {
            const size_t kc = F / w;
            unsigned char* wd = copy2d(b[10] + (size_t)r * kc, kc, D, F);
            unsigned char* sd = copy2d(b[11] + (size_t)r * (GF / w) * 2, (GF / w) * 2, D, GF * 2);
            L.down = {wd, reinterpret_cast<const uint16_t*>(sd), (int)D, (int)kc};
        }
    }
    return ce == cudaSuccess ? AF_OK : af::cuda_fail(ce, "af_engine_create_tp: weights");
}

// Reads the file into the device arena and points every tensor into it.
// Block order (weight_loader.h next_block, engine.cu:103-147): embedding FP32
// [V, D]; per layer: input norm FP32 [D], post-attention norm FP32 [D], then qkv,
// o, gate, up, down as FP8 weights [N, K] each followed by FP16 group scales
// [N, K/128]; final norm FP32 [D]; lm_head FP16 [V, D].
af_status load_file(af_engine* e, const char* path) {
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return AF_ERR_INVALID;
    struct stat sb;
    if (fstat(fd, &sb) != 0 || (size_t)sb.st_size < kAlign) {
        close(fd);
        return AF_ERR_INVALID;
    }
    const size_t size = (size_t)sb.st_size;
    void* map = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) return AF_ERR_INVALID;
    const unsigned char* f = static_cast<const unsigned char*>(map);
    Header& h = e->h;
    std::memcpy(&h, f, sizeof(Header));
    af_status st = AF_OK;
    if (std::memcmp(h.magic, "ATOM", 4) != 0 || h.version != 1 || h.group_size != kGroup || h.dim <= 0 ||
        h.ffn <= 0 || h.n_layers <= 0 || h.n_heads <= 0 || h.n_kv_heads <= 0 || h.vocab <= 0 ||
        h.dim % h.n_heads != 0 || h.n_heads % h.n_kv_heads != 0 || h.dim % kGroup != 0 || h.ffn % kGroup != 0)
        st = AF_ERR_INVALID;
    e->HD = st == AF_OK ? h.dim / h.n_heads : 0;
    e->QD = h.n_heads * e->HD;
    e->KVD = h.n_kv_heads * e->HD;
    e->QKV = e->QD + 2 * e->KVD;
    // the block plan, and the size the file must have
    size_t off = kAlign;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off += pad(bytes);
        return o;
    };
    struct Plan {
        size_t embed, final_norm, lm_head;
        std::vector<size_t> blocks;   // per layer: in_norm, post_norm, then (w, s) x 5
    } plan;
    const size_t D = h.dim, F = h.ffn, V = h.vocab;
    plan.embed = take(V * D * 4);
    const int NK[5][2] = {{e->QKV, h.dim}, {h.dim, h.dim}, {h.ffn, h.dim}, {h.ffn, h.dim}, {h.dim, h.ffn}};
    for (int l = 0; st == AF_OK && l < h.n_layers; ++l) {
        plan.blocks.push_back(take(D * 4));
        plan.blocks.push_back(take(D * 4));
        for (auto& nk : NK) {
            plan.blocks.push_back(take((size_t)nk[0] * nk[1]));
            plan.blocks.push_back(take((size_t)nk[0] * (nk[1] / kGroup) * 2));
        }
    }
    plan.final_norm = take(D * 4);
    plan.lm_head = take(V * D * 2);
    (void)F;
    if (st == AF_OK && size < off) st = AF_ERR_INVALID;
    // this rank's part of the model (the whole model when world == 1)
    const int w = e->world;
    if (st == AF_OK && (h.n_heads % w || h.n_kv_heads % w || h.ffn % (kGroup * w) || h.dim % (kGroup * w)))
        st = AF_ERR_UNSUPPORTED;   // heads, FFN rows and K shards must split evenly into whole scale groups
    e->NHl = h.n_heads / w;
    e->NKVl = h.n_kv_heads / w;
    e->FFNl = h.ffn / w;
    e->v0 = (int)((long long)e->rank * h.vocab / w);
    e->v1 = (int)((long long)(e->rank + 1) * h.vocab / w);
    e->QD = e->NHl * e->HD;
    e->KVD = e->NKVl * e->HD;
    e->QKV = e->QD + 2 * e->KVD;
    if (st == AF_OK && e->world > 1) {
        e->file_bytes = off;
        st = load_shards(e, f, plan.embed, plan.final_norm, plan.lm_head, plan.blocks);
        munmap(map, size);
        return st;
    }
    if (st == AF_OK) {
        e->file_bytes = off;
        cudaError_t ce = cudaMalloc(&e->arena, off - kAlign);
        // copy in pieces (the source is a file mapping)
        for (size_t o = kAlign; ce == cudaSuccess && o < off; o += (256u << 20)) {
            const size_t n = off - o < (256u << 20) ? off - o : (256u << 20);
            ce = cudaMemcpy(e->arena + (o - kAlign), f + o, n, cudaMemcpyHostToDevice);
        }
        if (ce != cudaSuccess) st = af::cuda_fail(ce, "af_engine_create: weights");
    }
    munmap(map, size);
    if (st != AF_OK) return st;
    auto at = [&](size_t o) { return e->arena + (o - kAlign); };
    e->embed = reinterpret_cast<const float*>(at(plan.embed));
    e->final_norm = reinterpret_cast<const float*>(at(plan.final_norm));
    e->lm_head = reinterpret_cast<const uint16_t*>(at(plan.lm_head));
    e->layers.resize(h.n_layers);
    for (int l = 0; l < h.n_layers; ++l) {
        const size_t* b = &plan.blocks[(size_t)l * 12];
        Layer& L = e->layers[l];
        L.in_norm = reinterpret_cast<const float*>(at(b[0]));
        L.post_norm = reinterpret_cast<const float*>(at(b[1]));
        Linear* lin[5] = {&L.qkv, &L.o, &L.gate, &L.up, &L.down};
        for (int i = 0; i < 5; ++i) {
            lin[i]->w = at(b[2 + 2 * i]);
            lin[i]->s = reinterpret_cast<const uint16_t*>(at(b[3 + 2 * i]));
            lin[i]->N = NK[i][0];
            lin[i]->K = NK[i][1];
        }
    }
    return AF_OK;
}

}  // namespace

namespace {

// One step's launches on the engine's stream.
af_status launch_step(af_engine* e, bool advance) {
    const Header& h = e->h;
    cudaStream_t st = e->stream;
    int n = 0;
    af_status r = af_embed_lookup(e->embed, e->d_token, e->x, h.dim, st);
    ++n;
    if (e->mode == AF_ENGINE_EXACT) {
        // chain segment s precedes layer s's attention; the last one follows the last layer's
        for (int l = 0; r == AF_OK && l <= h.n_layers; ++l) {
            const std::vector<af_chain_op>& seg = e->segments[l];
            r = af_gemv_chain(seg.data(), (int)seg.size(), e->chain_ws, e->chain_ws_bytes, st);
            ++n;
            if (r == AF_OK && l < h.n_layers) {
                Layer& L = e->layers[l];
                r = af_decode_rope_attention(e->qkv, e->cos_tab, e->sin_tab, e->d_pos, L.k_cache, L.v_cache, e->attn,
                                             e->NHl, e->NKVl, e->HD, e->max_seq, e->attn_ws, e->attn_ws_bytes,
                                             st);
                ++n;
            }
        }
    } else {
        for (int l = 0; r == AF_OK && l < h.n_layers; ++l) {
            Layer& L = e->layers[l];
            r = af_rmsnorm_w8a16_gemv(e->x, L.in_norm, kNormEps, L.qkv.w, L.qkv.s, e->qkv, L.qkv.N, L.qkv.K, kGroup,
                                      AF_SCALE_GROUP_F16, nullptr, st);
            if (r == AF_OK)
                r = af_decode_rope_attention_fast(e->qkv, e->cos_tab, e->sin_tab, e->d_pos, L.k_cache, L.v_cache,
                                                  e->attn, e->NHl, e->NKVl, e->HD, e->max_seq, e->attn_ws,
                                                  e->attn_ws_bytes, st);
            if (r == AF_OK)
                r = e->comm ? af_w8a16_gemv_allreduce_residual(e->attn, L.o.w, L.o.s, e->x, L.o.N, L.o.K, kGroup,
                                                               AF_SCALE_GROUP_F16, e->comm, st)
                            : af_w8a16_gemv_residual(e->attn, L.o.w, L.o.s, e->x, L.o.N, L.o.K, kGroup,
                                                     AF_SCALE_GROUP_F16, nullptr, st);
            if (r == AF_OK)
                r = af_rmsnorm_w8a16_swiglu(e->x, L.post_norm, kNormEps, L.gate.w, L.gate.s, L.up.w, L.up.s, e->hbuf,
                                            L.gate.N, L.gate.K, kGroup, AF_SCALE_GROUP_F16, nullptr, nullptr, st);
            if (r == AF_OK)
                r = e->comm ? af_w8a16_gemv_allreduce_residual(e->hbuf, L.down.w, L.down.s, e->x, L.down.N,
                                                               L.down.K, kGroup, AF_SCALE_GROUP_F16, e->comm, st)
                            : af_w8a16_gemv_residual(e->hbuf, L.down.w, L.down.s, e->x, L.down.N, L.down.K, kGroup,
                                                     AF_SCALE_GROUP_F16, nullptr, st);
            n += 5;
        }
    }
    if (r == AF_OK) r = af_rmsnorm(e->x, e->final_norm, kNormEps, e->xn, h.dim, st);
    if (r == AF_OK)
        r = e->comm ? af_lm_head_gemv_tp(e->xn, e->lm_head, AF_W_F16, nullptr, e->logits, e->v1 - e->v0, h.dim, e->v0,
                                         e->d_token, e->amode, e->lm_ws, e->lm_ws_bytes, e->comm, st)
                    : af_lm_head_gemv(e->xn, e->lm_head, AF_W_F16, nullptr, e->logits, h.vocab, h.dim, e->d_token,
                                      e->amode, e->lm_ws, e->lm_ws_bytes, st);
    n += 2;
    if (r == AF_OK && advance) r = af_decode_advance(e->d_pos, 1, st);
    e->launches = n;
    return r;
}

// The exact mode's chain segments: segment 0 is layer 0's RMSNorm + QKV; segment
// l + 1 is layer l's O + residual, RMSNorm + gate/up + SwiGLU, down + residual,
// and layer l + 1's RMSNorm + QKV -- each op waiting for the one before.
void build_segments(af_engine* e) {
    const Header& h = e->h;
    auto qkv_op = [&](int l) {
        const Layer& L = e->layers[l];
        af_chain_op op{};
        op.kind = AF_OP_RMSNORM_GEMV;
        op.N = L.qkv.N;
        op.K = L.qkv.K;
        op.wait_prev = 1;
        op.x = e->x;
        op.w = L.qkv.w;
        op.scales = L.qkv.s;
        op.norm_w = L.in_norm;
        op.eps = kNormEps;
        op.y = e->qkv;
        return op;
    };
    e->segments.assign(h.n_layers + 1, {});
    e->segments[0].push_back(qkv_op(0));
    for (int l = 0; l < h.n_layers; ++l) {
        const Layer& L = e->layers[l];
        std::vector<af_chain_op>& seg = e->segments[l + 1];
        af_chain_op o{};
        o.kind = AF_OP_GEMV_RESIDUAL;
        o.N = L.o.N;
        o.K = L.o.K;
        o.x = e->attn;
        o.w = L.o.w;
        o.scales = L.o.s;
        o.y = e->x;
        seg.push_back(o);
        af_chain_op gu{};
        gu.kind = AF_OP_RMSNORM_SWIGLU;
        gu.N = L.gate.N;
        gu.K = L.gate.K;
        gu.wait_prev = 1;
        gu.x = e->x;
        gu.w = L.gate.w;
        gu.scales = L.gate.s;
        gu.w2 = L.up.w;
        gu.scales2 = L.up.s;
        gu.norm_w = L.post_norm;
        gu.eps = kNormEps;
        gu.y = e->hbuf;
        seg.push_back(gu);
        af_chain_op dn{};
        dn.kind = AF_OP_GEMV_RESIDUAL;
        dn.N = L.down.N;
        dn.K = L.down.K;
        dn.wait_prev = 1;
        dn.x = e->hbuf;
        dn.w = L.down.w;
        dn.scales = L.down.s;
        dn.y = e->x;
        seg.push_back(dn);
        if (l + 1 < h.n_layers) seg.push_back(qkv_op(l + 1));
    }
}

}  // namespace

extern "C" af_status af_engine_destroy(af_engine* e) {
    if (e == nullptr) return AF_ERR_INVALID;
    if (e->graph) cudaGraphExecDestroy(e->graph);
    if (e->stream) cudaStreamSynchronize(e->stream);
    for (void* p : e->owned) cudaFree(p);
    cudaFree(e->arena);
    cudaFree(e->acts);
    cudaFree(e->kv);
    if (e->stream) cudaStreamDestroy(e->stream);
    delete e;
    return AF_OK;
}

static af_status engine_create(const char* bin_path, int max_seq, af_engine_mode mode, af_argmax_mode argmax_mode,
                               af_tp_comm* comm, af_engine** out) {
    if (bin_path == nullptr || out == nullptr || max_seq <= 0) return AF_ERR_INVALID;
    if (mode != AF_ENGINE_EXACT && mode != AF_ENGINE_FAST) return AF_ERR_INVALID;
    if (argmax_mode != AF_ARGMAX_TRUE && argmax_mode != AF_ARGMAX_REF_COMPAT) return AF_ERR_INVALID;
    *out = nullptr;
    af_engine* e = new af_engine();
    if (comm != nullptr) {
        int dev = -1;
        if (cudaGetDevice(&dev) != cudaSuccess || dev != comm->device) {
            delete e;
            return AF_ERR_INVALID;   // the engine runs on the communicator's device
        }
        e->comm = comm->world > 1 ? comm : nullptr;
        e->rank = comm->rank;
        e->world = comm->world;
    }
    e->max_seq = max_seq;
    e->mode = mode;
    e->amode = argmax_mode;
    af_status st = load_file(e, bin_path);
    const Header& h = e->h;
    if (st == AF_OK && e->HD != 128) st = AF_ERR_UNSUPPORTED;   // the attention kernels' head dim
    if (st == AF_OK) {
        cudaError_t ce = cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking);
        if (ce != cudaSuccess) st = af::cuda_fail(ce, "af_engine_create: stream");
    }
    if (st == AF_OK) {
        // activations, state and workspaces: one arena, 256-byte aligned pieces
        e->attn_ws_bytes = af_decode_attention_workspace_bytes(e->NHl, e->NKVl, max_seq);
        e->lm_ws_bytes = af_lm_head_workspace_bytes(e->v1 - e->v0, h.dim, AF_W_F16);
        e->chain_ws_bytes = af_chain_workspace_bytes(4);
        const size_t half_tab = (size_t)max_seq * (e->HD / 2) * 4;
        const size_t sizes[] = {(size_t)h.dim * 2, (size_t)h.dim * 2, (size_t)e->QKV * 2, (size_t)e->QD * 2,
                                (size_t)e->FFNl * 2, (size_t)(e->v1 - e->v0) * 4, 4, 4, half_tab, half_tab,
                                e->attn_ws_bytes, e->lm_ws_bytes, e->chain_ws_bytes};
        size_t total = 0;
        for (size_t b : sizes) total += pad(b);
        cudaError_t ce = cudaMalloc(&e->acts, total);
        if (ce == cudaSuccess) ce = cudaMemsetAsync(e->acts, 0, total, e->stream);
        if (ce == cudaSuccess) {
            const size_t kvb = (size_t)h.n_layers * 2 * max_seq * e->KVD * 2;
            ce = cudaMalloc(&e->kv, kvb);
            if (ce == cudaSuccess) ce = cudaMemsetAsync(e->kv, 0, kvb, e->stream);
        }
        if (ce != cudaSuccess) st = af::cuda_fail(ce, "af_engine_create: arenas");
        if (st == AF_OK) {
            unsigned char* p = e->acts;
            void* ptrs[13];
            for (int i = 0; i < 13; ++i) {
                ptrs[i] = p;
                p += pad(sizes[i]);
            }
            e->x = static_cast<__half*>(ptrs[0]);
            e->xn = static_cast<__half*>(ptrs[1]);
            e->qkv = static_cast<__half*>(ptrs[2]);
            e->attn = static_cast<__half*>(ptrs[3]);
            e->hbuf = static_cast<__half*>(ptrs[4]);
            e->logits = static_cast<float*>(ptrs[5]);
            e->d_token = static_cast<int*>(ptrs[6]);
            e->d_pos = static_cast<int*>(ptrs[7]);
            e->cos_tab = static_cast<float*>(ptrs[8]);
            e->sin_tab = static_cast<float*>(ptrs[9]);
            e->attn_ws = ptrs[10];
            e->lm_ws = ptrs[11];
            e->chain_ws = ptrs[12];
            for (int l = 0; l < h.n_layers; ++l) {
                __half* base = reinterpret_cast<__half*>(e->kv) + (size_t)l * 2 * max_seq * e->KVD;
                e->layers[l].k_cache = base;
                e->layers[l].v_cache = base + (size_t)max_seq * e->KVD;
            }
            // RoPE tables: the reference's host formula (helpers.cu build_rope_cache)
            std::vector<float> cs((size_t)max_seq * (e->HD / 2)), sn(cs.size());
            st = af_rope_tables(cs.data(), sn.data(), max_seq, e->HD, kRopeBase);
            if (st == AF_OK) {
                ce = cudaMemcpyAsync(e->cos_tab, cs.data(), half_tab, cudaMemcpyHostToDevice, e->stream);
                if (ce == cudaSuccess)
                    ce = cudaMemcpyAsync(e->sin_tab, sn.data(), half_tab, cudaMemcpyHostToDevice, e->stream);
                if (ce == cudaSuccess) ce = cudaStreamSynchronize(e->stream);
                if (ce != cudaSuccess) st = af::cuda_fail(ce, "af_engine_create: tables");
            }
            build_segments(e);
        }
    }
    if (st == AF_OK && e->comm != nullptr && e->comm->nmax < h.dim) st = AF_ERR_INVALID;   // all-reduce rows
    if (st != AF_OK) {
        af_engine_destroy(e);
        return st;
    }
    *out = e;
    return AF_OK;
}

extern "C" af_status af_engine_create(const char* bin_path, int max_seq, af_engine_mode mode, af_argmax_mode argmax_mode,
                                      af_engine** out) {
    return engine_create(bin_path, max_seq, mode, argmax_mode, nullptr, out);
}

extern "C" af_status af_engine_create_tp(const char* bin_path, int max_seq, af_argmax_mode argmax_mode,
                                         af_tp_comm* comm, af_engine** out) {
    if (comm == nullptr) return AF_ERR_INVALID;
    for (int r = 0; r < comm->world; ++r)
        if (comm->peer[r] == nullptr) return AF_ERR_INVALID;   // peers not opened
    return engine_create(bin_path, max_seq, AF_ENGINE_FAST, argmax_mode, comm, out);
}

extern "C" af_status af_engine_info(const af_engine* e, int* dims) {
    if (e == nullptr || dims == nullptr) return AF_ERR_INVALID;
    const Header& h = e->h;
    const int v[9] = {h.dim, h.ffn, h.n_layers, h.n_heads, h.n_kv_heads, h.vocab, e->max_seq, e->launches,
                      (int)(e->file_bytes >> 20)};
    for (int i = 0; i < 9; ++i) dims[i] = v[i];
    return AF_OK;
}

extern "C" af_status af_engine_set_position(af_engine* e, int pos) {
    if (e == nullptr || pos < 0 || pos >= e->max_seq) return AF_ERR_INVALID;
    cudaError_t ce = cudaMemcpyAsync(e->d_pos, &pos, 4, cudaMemcpyHostToDevice, e->stream);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(e->stream);   // pos is a host local
    return ce == cudaSuccess ? AF_OK : af::cuda_fail(ce, "af_engine_set_position");
}

extern "C" af_status af_engine_get_position(af_engine* e, int* pos) {
    if (e == nullptr || pos == nullptr) return AF_ERR_INVALID;
    cudaError_t ce = cudaMemcpyAsync(pos, e->d_pos, 4, cudaMemcpyDeviceToHost, e->stream);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(e->stream);
    return ce == cudaSuccess ? AF_OK : af::cuda_fail(ce, "af_engine_get_position");
}

extern "C" af_status af_engine_inject_token(af_engine* e, int token) {
    if (e == nullptr || token < 0 || token >= e->h.vocab) return AF_ERR_INVALID;
    cudaError_t ce = cudaMemcpyAsync(e->d_token, &token, 4, cudaMemcpyHostToDevice, e->stream);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(e->stream);   // token is a host local
    return ce == cudaSuccess ? AF_OK : af::cuda_fail(ce, "af_engine_inject_token");
}

extern "C" af_status af_engine_output_token(af_engine* e, int* token) {
    if (e == nullptr || token == nullptr) return AF_ERR_INVALID;
    cudaError_t ce = cudaMemcpyAsync(token, e->d_token, 4, cudaMemcpyDeviceToHost, e->stream);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(e->stream);
    return ce == cudaSuccess ? AF_OK : af::cuda_fail(ce, "af_engine_output_token");
}

extern "C" af_status af_engine_step(af_engine* e, int advance) {
    if (e == nullptr) return AF_ERR_INVALID;
    if (!e->stepped) {
        // workspaces start at zero (every kernel leaves them so)
        cudaError_t ce = cudaMemsetAsync(e->attn_ws, 0, e->attn_ws_bytes, e->stream);
        if (ce == cudaSuccess) ce = cudaMemsetAsync(e->lm_ws, 0, e->lm_ws_bytes, e->stream);
        if (ce == cudaSuccess) ce = cudaMemsetAsync(e->chain_ws, 0, e->chain_ws_bytes, e->stream);
        if (ce != cudaSuccess) return af::cuda_fail(ce, "af_engine_step");
    }
    af_status st = launch_step(e, advance != 0);
    if (st == AF_OK) e->stepped = true;
    return st;
}

extern "C" af_status af_engine_capture(af_engine* e, int advance) {
    if (e == nullptr) return AF_ERR_INVALID;
    if (!e->stepped) return AF_ERR_INVALID;   // the first step is eager (kernel attributes, workspaces)
    cudaError_t ce = cudaStreamSynchronize(e->stream);
    if (ce != cudaSuccess) return af::cuda_fail(ce, "af_engine_capture");
    if (e->graph) {
        cudaGraphExecDestroy(e->graph);
        e->graph = nullptr;
    }
    cudaGraph_t g = nullptr;
    ce = cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal);
    if (ce != cudaSuccess) return af::cuda_fail(ce, "af_engine_capture: begin");
    const af_status st = launch_step(e, advance != 0);
    ce = cudaStreamEndCapture(e->stream, &g);
    if (st != AF_OK) {
        if (g) cudaGraphDestroy(g);
        return st;
    }
    if (ce == cudaSuccess) ce = cudaGraphInstantiate(&e->graph, g, 0);
    if (g) cudaGraphDestroy(g);
    return ce == cudaSuccess ? AF_OK : af::cuda_fail(ce, "af_engine_capture");
}

extern "C" af_status af_engine_replay(af_engine* e, int n) {
    if (e == nullptr || e->graph == nullptr || n < 0) return AF_ERR_INVALID;
    for (int i = 0; i < n; ++i) {
        cudaError_t ce = cudaGraphLaunch(e->graph, e->stream);
        if (ce != cudaSuccess) return af::cuda_fail(ce, "af_engine_replay");
    }
    return AF_OK;
}

extern "C" af_status af_engine_synchronize(af_engine* e) {
    if (e == nullptr) return AF_ERR_INVALID;
    cudaError_t ce = cudaStreamSynchronize(e->stream);
    return ce == cudaSuccess ? AF_OK : af::cuda_fail(ce, "af_engine_synchronize");
}

extern "C" void* af_engine_stream(af_engine* e) { return e ? e->stream : nullptr; }
extern "C" int* af_engine_device_token(af_engine* e) { return e ? e->d_token : nullptr; }
extern "C" int* af_engine_device_position(af_engine* e) { return e ? e->d_pos : nullptr; }
extern "C" const float* af_engine_logits(af_engine* e) { return e ? e->logits : nullptr; }
