// A whole decoder on the hot path's kernels: the launches the reference's
// graph builds (plainsight-systems/charlotte, src/core/graph/graph.cpp:
// Builder::embed :155, attention :159-230, gated_feed_forward :232-262,
// output :264-292; the architectures' orders in src/core/arch/{qwen3,llama,
// gemma3}), each step in that order on one stream, every launch with
// programmatic dependent launch.
//
// Buffers follow the reference's working set (graph.cpp decoder_working_set:
// hidden, normed, query, key, value, attention, partials, partial_stats,
// output, activation, logits, the selection's partials, candidates,
// sampled) sized for a step of max_step_tokens; an f16 KV cache per layer of
// `context` slots, or, for a sliding-window layer, a ring of window + step
// slots (src/core/cache/kv.h:13-34: position p in slot p mod slots).
//
// Decode: the step's position lives in a device word and its one token is
// the last draw's (gather's fed form), so a decode step is captured once as
// a CUDA graph and replayed; a closing launch records the drawn token and
// advances the position.
//
// Batched decode (no counterpart in the reference, which runs one sequence):
// a decoder may hold S sequences, each with its own caches (sequence s's at
// s·stride in each layer's cache allocation). A prompt step runs one
// sequence's tokens; a batched step runs one token of every sequence, all at
// the same position, as S rows — the products take the S rows in one pass of
// the weights (a row's bits are those it has alone), rope, attention and the
// selection treat each row as its own sequence.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <new>
#include <vector>

#include "api_common.h"
#include "charlotte_b200.h"
#include "formats.cuh"
#include "kernels.h"
#include "matmul.h"

namespace cb {

namespace {

struct DevWeight {
    uint8_t* piece = nullptr;
    uint32_t format = 0, rows = 0, cols = 0, blocks = 0;
};

struct DevLayer {
    float* attn_norm = nullptr;
    DevWeight q, k, v, o, gate, up, down;
    float* q_norm = nullptr;
    float* k_norm = nullptr;
    float* post_attn_norm = nullptr;
    float* ffn_norm = nullptr;
    float* post_ffn_norm = nullptr;
    float* turns = nullptr;
    uint16_t* key_cache = nullptr;    // [sequences][slots][kv_heads][head_dim]
    uint16_t* value_cache = nullptr;
    uint32_t window = 0, slots = 0;
    uint64_t sequence_stride = 0;      // elements between sequences' caches
    // CB_DECODER_TENSOR_PREFILL: each product's weights densified to f16
    // once at creation (cb_matmul_densify), read by its tensor-form steps.
    void* dense_qkv = nullptr;
    void* dense_o = nullptr;
    void* dense_gate_up = nullptr;
    void* dense_down = nullptr;
};

// Records each row's drawn token and advances the step's position (decode
// graph): step i's tokens at [i·rows, (i+1)·rows).
__global__ void advance_kernel(uint32_t* state, const uint32_t* sampled, uint32_t* tokens_out, uint32_t* failed_out,
                               uint32_t capacity, uint32_t rows) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint32_t step = state[1];
    for (uint32_t r = threadIdx.x; r < rows; r += blockDim.x) {
        if (step < capacity) {
            tokens_out[static_cast<size_t>(step) * rows + r] = sampled[4u * r];
            failed_out[static_cast<size_t>(step) * rows + r] = sampled[4u * r + 1u];
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        state[0] += 1u;   // position
        state[1] = step + 1u;
    }
}

}  // namespace

}  // namespace cb

struct cb_decoder {
    cb_model model{};
    uint32_t max_tokens = 0;
    uint32_t max_chunks = 0;
    int sms = 0;
    cudaStream_t stream = nullptr;
    std::vector<void*> allocations;
    cb::DevWeight token_embd, output;
    float* output_norm = nullptr;
    float* factors = nullptr;
    std::vector<cb::DevLayer> layers;
    // working set
    float *hidden = nullptr, *normed = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr;
    float *out = nullptr, *act = nullptr, *logits = nullptr, *partials = nullptr, *stats = nullptr;
    unsigned int* tickets = nullptr;
    uint32_t* sel_partials = nullptr;
    unsigned int* sel_ticket = nullptr;
    uint32_t* candidates = nullptr;
    uint32_t* sampled = nullptr;
    uint32_t* ids = nullptr;
    uint32_t* state = nullptr;       // [0] position, [1] decode step index
    uint32_t* gen_tokens = nullptr;  // generate's drawn tokens
    uint32_t* gen_failed = nullptr;
    uint32_t gen_capacity = 0;
    cudaGraphExec_t decode_graph = nullptr;   // fed step + advance (generate)
    cb_sampling graph_sampling{};
    cudaGraphExec_t step_graph = nullptr;     // one host-fed token with logits (step)
    cb_sampling step_sampling{};
    bool has_step = false;
    uint32_t next_position = 0;   // the position after the last step's tokens
    uint32_t sequences = 1;
    uint32_t rows = 0;            // working-set rows: max(step tokens, sequences)
    std::vector<uint32_t> seq_next;   // each sequence's position after its last step
    std::vector<uint8_t> seq_drawn;   // whether a sequence's last step drew a token
    bool tensor_prefill = false;  // CB_DECODER_TENSOR_PREFILL
    float* hidden2 = nullptr;
    void* tensor_scratch = nullptr;
    uint64_t tensor_scratch_bytes = 0;
    // f16 copies a tensor-form step's producers write for the next product
    // (its x16): the norms' rows, the attention's output, gate|up's output.
    void* normed16 = nullptr;
    void* att16 = nullptr;
    void* act16 = nullptr;
    void* split_scratch = nullptr;   // the split form's range sums (few-tile, wide-K products)
    uint64_t split_scratch_bytes = 0;
};

namespace {

using namespace cb;

template <typename T>
int dalloc(cb_decoder* d, T** p, size_t count) {
    void* q = nullptr;
    const cudaError_t e = cudaMalloc(&q, count * sizeof(T) > 0 ? count * sizeof(T) : 16);
    if (e != cudaSuccess) return fail_cuda(e, "cb_decoder_create: cudaMalloc");
    d->allocations.push_back(q);
    *p = static_cast<T*>(q);
    return CB_OK;
}

int upload_f32(cb_decoder* d, float** dst, const float* host, size_t n) {
    if (!host) { *dst = nullptr; return CB_OK; }
    if (int rc = dalloc(d, dst, n)) return rc;
    const cudaError_t e = cudaMemcpy(*dst, host, n * sizeof(float), cudaMemcpyHostToDevice);
    return e == cudaSuccess ? CB_OK : fail_cuda(e, "cb_decoder_create: upload");
}

uint32_t weights_per_block(uint32_t f) {
    return f == CB_Q6_K ? 256u : (f == CB_Q4_0 || f == CB_Q4_1 || f == CB_Q8_0 ? 32u : 1u);
}

int upload_weight(cb_decoder* d, DevWeight* w, const cb_weight& src, const char* name) {
    if (src.rows == 0) return CB_OK;
    if (src.format != CB_Q4_0 && src.format != CB_Q4_1 && src.format != CB_Q8_0 && src.format != CB_Q6_K &&
        src.format != CB_BF16)
        return fail(CB_ERROR_BUILD, "cb_decoder_create: %s's format %u has no matmul kernel", name, src.format);
    if (src.cols % weights_per_block(src.format) != 0)
        return fail(CB_ERROR_BUILD, "cb_decoder_create: %s's rows of %u are not whole blocks", name, src.cols);
    if (!src.stored_host) return fail(CB_ERROR_BUILD, "cb_decoder_create: %s has no data", name);
    const uint64_t blocks = static_cast<uint64_t>(src.rows) * src.cols / weights_per_block(src.format);
    if (blocks > 0xFFFFFFFFull) return fail(CB_ERROR_BUILD, "cb_decoder_create: %s is too large for one piece", name);
    const size_t bytes = cb_piece_bytes(src.format, blocks);
    std::vector<uint8_t> host(bytes);
    if (int rc = cb_piece_from_stored(src.format, src.stored_host, blocks, host.data())) return rc;
    if (int rc = dalloc(d, &w->piece, bytes)) return rc;
    const cudaError_t e = cudaMemcpy(w->piece, host.data(), bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return fail_cuda(e, "cb_decoder_create: upload");
    w->format = src.format;
    w->rows = src.rows;
    w->cols = src.cols;
    w->blocks = static_cast<uint32_t>(blocks);
    return CB_OK;
}

cb_member member_of(const DevWeight& w) { return {w.piece, w.blocks, 0, w.rows, 0}; }

int launched(cudaError_t e, const char* what) { return e == cudaSuccess ? CB_OK : fail_cuda(e, what); }

// Steps of this many tokens or more take the tensor form under
// CB_DECODER_TENSOR_PREFILL.
constexpr uint32_t kDecoderTensorTokens = 128;

// A product's description: its members, epilogue and activation.
cb_matmul description(const cb_decoder* d, std::initializer_list<const DevWeight*> ws, uint32_t epilogue) {
    cb_matmul m{};
    const DevWeight* first = *ws.begin();
    m.format = first->format;
    m.columns = first->cols;
    m.members = static_cast<uint32_t>(ws.size());
    m.epilogue = epilogue;
    m.activation = d->model.activation;
    uint32_t i = 0;
    for (const DevWeight* w : ws) m.member[i++] = member_of(*w);
    return m;
}

// One matmul launch through the same path as cb_matmul_run; `dense`: the
// product's densified weights for the tensor form (or NULL).
// `x16`/`out16`: the dense form's f16 copy of x (written by the producer)
// and of a gated output (for the next product), or NULL.
int product(cb_decoder* d, std::initializer_list<const DevWeight*> ws, uint32_t epilogue, const float* x,
            uint32_t x_stride, uint32_t tokens, float* const outs[3], const uint32_t strides[3],
            const void* dense = nullptr, const void* x16 = nullptr, void* out16 = nullptr) {
    cb_matmul m = description(d, ws, epilogue);
    uint32_t flags = CB_MATMUL_PDL;
    if (d->tensor_prefill && tokens >= kDecoderTensorTokens) {
        flags |= CB_MATMUL_TENSOR;
        m.scratch = d->tensor_scratch;
        m.scratch_bytes = d->tensor_scratch_bytes;
        m.dense = dense;
        m.x16 = dense ? x16 : nullptr;
        m.out16 = dense ? out16 : nullptr;
    } else if (tokens > 1) {
        // range-sum scratch: cb_matmul_run takes the split form where it pays
        m.scratch = d->split_scratch;
        m.scratch_bytes = d->split_scratch_bytes;
    }
    return cb_matmul_run(&m, x, x_stride, tokens, outs, strides, flags, d->stream);
}

// A one-token product with the RMSNorm before it folded into its prologue
// (matmul_decode.cu): every CTA computes the normed row of hidden (+ y,
// post-normed first when post_gain); CTA 0 writes hidden + y to hidden_out.
int product_normed(cb_decoder* d, std::initializer_list<const DevWeight*> ws, uint32_t epilogue, float* const outs[3],
                   const float* hidden, const float* y, const float* post_gain, const float* gain, float* hidden_out) {
    MatmulArgs a{};
    const DevWeight* first = *ws.begin();
    a.format = first->format;
    a.columns = first->cols;
    a.members = static_cast<uint32_t>(ws.size());
    a.epilogue = epilogue;
    a.activation = d->model.activation;
    a.tokens = 1;
    uint32_t i = 0, total = 0;
    for (const DevWeight* w : ws) {
        a.member[i++] = {w->piece, w->blocks, 0, w->rows, 0};
        total += w->rows;
    }
    a.total_rows = epilogue == CB_EPILOGUE_GATED ? first->rows : total;
    for (uint32_t k = 0; k < 3; ++k) a.out[k] = outs[k];
    a.x_stride = a.columns;
    a.fault = fault_word();
    a.norm_hidden = hidden;
    a.norm_y = y;
    a.norm_post_gain = post_gain;
    a.norm_gain = gain;
    a.norm_hidden_out = hidden_out;
    a.norm_epsilon = d->model.epsilon;
    return launched(matmul_decode(a, d->sms, d->stream, true), "step: normed product");
}

// The step's launches (graph.cpp's order). `fed`: the token is the last
// draw. `seq` >= 0: `tokens` consecutive positions of sequence `seq`; -1:
// a batched step, row r the token of sequence r (tokens == sequences).
int enqueue_step(cb_decoder* d, uint32_t tokens, bool fed, bool logits, const cb_sampling& s, int seq = 0,
                 bool head_and_draw = true) {
    const bool batch = seq < 0;
    const uint32_t row0 = batch ? 0u : static_cast<uint32_t>(seq);   // this step's record / logits row
    const cb_model& m = d->model;
    const uint32_t H = m.hidden, dh = m.head_dim, qd = m.query_heads * dh, kvd = m.kv_heads * dh;
    const uint32_t* pos = d->state;
    // embed
    {
        cb_gather g{};
        g.piece = d->token_embd.piece;
        g.format = d->token_embd.format;
        g.blocks = d->token_embd.blocks;
        g.width = H;
        g.first_row = 0;
        g.row_count = d->token_embd.rows;
        g.ids = d->ids;
        g.sampled = d->sampled + 4u * row0;
        g.fed = fed ? 1u : 0u;
        g.fed_stride = batch ? 4u : 0u;
        g.tokens = tokens;
        g.scale = m.embed_scale;
        g.hidden = d->hidden;
        if (int rc = launched(gather_run(g, d->stream, true), "step: gather")) return rc;
    }
    const float* pending_post = nullptr;
    bool pending_add = false;
    // A one-token step of one sequence folds each norm into the product after
    // it; the residual stream then alternates between two buffers.
    const bool fold = tokens == 1 && !batch;
    // A step whose products take the tensor form: its producers also write
    // f16 copies of the products' inputs.
    const bool tensor_step = d->tensor_prefill && tokens >= kDecoderTensorTokens;
    float* stream_buf[2] = {d->hidden, d->hidden2};
    uint32_t cur = 0;
    for (uint32_t l = 0; l < m.layers; ++l) {
        const DevLayer& L = d->layers[l];
        if (fold) {
            float* outs[3] = {d->q, d->k, d->v};
            if (int rc = product_normed(d, {&L.q, &L.k, &L.v}, CB_EPILOGUE_QKV, outs, stream_buf[cur],
                                        pending_add ? d->out : nullptr, pending_post, L.attn_norm,
                                        pending_add ? stream_buf[cur ^ 1u] : nullptr))
                return rc;
            if (pending_add) cur ^= 1u;
        } else {
            cb_norm n{d->hidden, d->out, L.attn_norm, pending_post, d->normed, H, tokens, pending_add ? 1u : 0u, 0u,
                      m.epsilon};
            n.normed16 = tensor_step ? d->normed16 : nullptr;
            if (int rc = launched(norm_run(n, d->stream, true), "step: attention norm")) return rc;
            float* outs[3] = {d->q, d->k, d->v};
            const uint32_t strides[3] = {qd, kvd, kvd};
            if (int rc = product(d, {&L.q, &L.k, &L.v}, CB_EPILOGUE_QKV, d->normed, H, tokens, outs, strides,
                                 L.dense_qkv, n.normed16))
                return rc;
        }
        cb_rope r{};
        r.query = d->q;
        r.key = d->k;
        r.value = d->v;
        const size_t cache_at = batch ? 0u : static_cast<size_t>(seq) * L.sequence_stride;
        r.key_cache = L.key_cache + cache_at;
        r.value_cache = L.value_cache + cache_at;
        r.rows_are_sequences = batch ? 1u : 0u;
        r.sequence_stride = L.sequence_stride;
        r.query_gain = L.q_norm;
        r.key_gain = L.k_norm;
        r.factors = d->factors;
        r.turns = L.turns;
        r.position = pos;
        r.tokens = tokens;
        r.head_dim = dh;
        r.query_heads = m.query_heads;
        r.kv_heads = m.kv_heads;
        r.halves = m.halves;
        r.slots = L.slots;
        r.epsilon = m.epsilon;
        // Decode shapes fold the rope into the attention's prologue (one
        // launch fewer a layer); steps of several positions launch it.
        const bool fuse_rope = tokens == 1u || batch;
        if (!fuse_rope)
            if (int rc = launched(rope_run(r, d->stream, true), "step: rope")) return rc;
        cb_attention at{};
        at.rope = fuse_rope ? &r : nullptr;
        at.query = d->q;
        at.key_cache = L.key_cache + cache_at;
        at.value_cache = L.value_cache + cache_at;
        at.rows_are_sequences = batch ? 1u : 0u;
        at.sequence_stride = L.sequence_stride;
        at.out = d->att;
        at.partials = d->partials;
        at.stats = d->stats;
        at.tickets = d->tickets;
        at.position = pos;
        at.tokens = tokens;
        at.head_dim = dh;
        at.query_heads = m.query_heads;
        at.kv_heads = m.kv_heads;
        at.slots = L.slots;
        at.window = L.window;
        at.max_chunks = d->max_chunks;
        at.scale_log2e = static_cast<float>(static_cast<double>(m.attention_scale) * 1.4426950408889634);
        const bool tensor_attention = tensor_step && attention_tensor_fits(at);
        if (tensor_attention) at.out16 = d->att16;
        if (int rc = launched(tensor_attention ? attention_tensor_run(at, d->stream, true) : attention_run(at, d->stream, true),
                              "step: attention"))
            return rc;
        {
            float* outs[3] = {d->out, nullptr, nullptr};
            const uint32_t strides[3] = {H, 0, 0};
            if (int rc = product(d, {&L.o}, CB_EPILOGUE_WRITE, d->att, qd, tokens, outs, strides, L.dense_o,
                                 at.out16))
                return rc;
        }
        if (fold) {
            float* outs[3] = {d->act, nullptr, nullptr};
            if (int rc = product_normed(d, {&L.gate, &L.up}, CB_EPILOGUE_GATED, outs, stream_buf[cur], d->out,
                                        L.post_attn_norm, L.ffn_norm, stream_buf[cur ^ 1u]))
                return rc;
            cur ^= 1u;
        } else {
            cb_norm n2{d->hidden, d->out, L.ffn_norm, L.post_attn_norm, d->normed, H, tokens, 1u, 0u, m.epsilon};
            n2.normed16 = tensor_step ? d->normed16 : nullptr;
            if (int rc = launched(norm_run(n2, d->stream, true), "step: feed-forward norm")) return rc;
            float* outs[3] = {d->act, nullptr, nullptr};
            const uint32_t strides[3] = {m.ffn, 0, 0};
            if (int rc = product(d, {&L.gate, &L.up}, CB_EPILOGUE_GATED, d->normed, H, tokens, outs, strides,
                                 L.dense_gate_up, n2.normed16, tensor_step ? d->act16 : nullptr))
                return rc;
        }
        {
            float* outs[3] = {d->out, nullptr, nullptr};
            const uint32_t strides[3] = {H, 0, 0};
            if (int rc = product(d, {&L.down}, CB_EPILOGUE_WRITE, d->act, m.ffn, tokens, outs, strides,
                                 L.dense_down, tensor_step && !fold ? d->act16 : nullptr))
                return rc;
        }
        pending_add = true;
        pending_post = L.post_ffn_norm;
    }
    if (!logits) return CB_OK;   // the residual stream is not carried to the next step
    // The output: a sequence step's last row, or every row of a batched step.
    const uint32_t heads = batch ? tokens : 1u;
    if (fold && head_and_draw) {
        const DevWeight& head = d->output.piece ? d->output : d->token_embd;
        float* outs[3] = {d->logits + static_cast<size_t>(row0) * m.vocab, nullptr, nullptr};
        if (int rc = product_normed(d, {&head}, CB_EPILOGUE_WRITE, outs, stream_buf[cur], d->out, pending_post,
                                    d->output_norm, nullptr))
            return rc;
    } else {
    if (fold) {
        // the caller wants the normed row (a vocabulary split): the norm kernel over the stream's buffer
        cb_norm fn{stream_buf[cur], d->out, d->output_norm, pending_post, d->normed, H, 1u, 1u, 1u, m.epsilon};
        if (int rc = launched(norm_run(fn, d->stream, true), "step: output norm")) return rc;
    } else {
        cb_norm fn{d->hidden, d->out, d->output_norm, pending_post, d->normed, H, tokens, 1u, batch ? 0u : 1u,
                   m.epsilon};
        if (int rc = launched(norm_run(fn, d->stream, true), "step: output norm")) return rc;
    }
    if (!head_and_draw) return CB_OK;   // the caller runs the head (a vocabulary split)
    {
        const DevWeight& head = d->output.piece ? d->output : d->token_embd;
        float* outs[3] = {d->logits + static_cast<size_t>(row0) * m.vocab, nullptr, nullptr};
        const uint32_t strides[3] = {m.vocab, 0, 0};
        const float* x = batch ? d->normed : d->normed + static_cast<size_t>(tokens - 1) * H;
        if (int rc = product(d, {&head}, CB_EPILOGUE_WRITE, x, H, heads, outs, strides)) return rc;
    }
    }
    cb_select sel{};
    sel.logits = d->logits + static_cast<size_t>(row0) * m.vocab;
    sel.count = m.vocab;
    sel.partials = d->sel_partials;
    sel.ticket = d->sel_ticket;
    sel.candidates = d->candidates + 128u * row0;
    sel.sampled = d->sampled + 4u * row0;
    sel.rows = heads;
    sel.logits_stride = m.vocab;
    sel.position = pos;
    sel.tokens = tokens;
    sel.seed0 = s.seed0;
    sel.seed1 = s.seed1;
    sel.top_k = s.top_k ? s.top_k : 1;
    sel.temperature = s.temperature;
    sel.top_p = s.top_p;
    sel.min_p = s.min_p;
    sel.log_min_p = s.min_p > 0.0f ? std::log(s.min_p) : 0.0f;
    return launched(select_run(sel, d->stream, true), "step: select");
}

bool same_sampling(const cb_sampling& a, const cb_sampling& b) { return std::memcmp(&a, &b, sizeof a) == 0; }

// Captures one decode step (one token, logits and draw) as a graph: fed
// (the token is the last draw) and closed by `advance` for generate, or
// reading its token from the ids buffer for a host-driven step.
int capture_step(cb_decoder* d, bool fed, const cb_sampling& smp, cudaGraphExec_t* out) {
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamBeginCapture(d->stream, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) return fail_cuda(e, "decoder: capture");
    // One token of the one sequence, or (several sequences) a batched step.
    const bool batch = d->sequences > 1;
    int rc = enqueue_step(d, batch ? d->sequences : 1u, fed, true, smp, batch ? -1 : 0);
    if (rc == CB_OK && fed) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(1);
        cfg.blockDim = dim3(d->sequences < 1024 ? (d->sequences + 31u) / 32u * 32u : 1024u);
        cfg.stream = d->stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, advance_kernel, d->state, static_cast<const uint32_t*>(d->sampled),
                               d->gen_tokens, d->gen_failed, d->gen_capacity, d->sequences);
        if (e != cudaSuccess) rc = fail_cuda(e, "decoder: advance");
    }
    const cudaError_t end = cudaStreamEndCapture(d->stream, &g);
    if (rc != CB_OK) { if (g) cudaGraphDestroy(g); return rc; }
    if (end != cudaSuccess) return fail_cuda(end, "decoder: end capture");
    e = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    return e == cudaSuccess ? CB_OK : fail_cuda(e, "decoder: instantiate");
}

// The end of a synchronous step: the fault word read and cleared. When a
// bounded wait ran out during the step, a CTA that gave up may not have
// taken its ticket, which would leave a ticket word part-counted and let
// the next step's fold start early; so the ticket words are cleared before
// the failure is reported, and the next step starts clean.
int finish_step(cb_decoder* d) {
    const int rc = cb_fault_check(nullptr);
    if (rc == CB_OK) return rc;
    const uint32_t S = d->sequences;
    const uint32_t tickets = std::max(cb_attention_tickets(d->rows, d->model.query_heads, d->model.kv_heads),
                                      S * d->model.kv_heads);
    cudaError_t e = cudaMemsetAsync(d->tickets, 0, tickets * sizeof(unsigned int), d->stream);
    if (e == cudaSuccess)
        e = cudaMemsetAsync(d->sel_ticket, 0,
                            static_cast<size_t>(S) * cb_select_tickets(d->model.vocab) * sizeof(unsigned int),
                            d->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(d->stream);
    return e == cudaSuccess ? rc : fail_cuda(e, "decoder: clearing the tickets after a failed step");
}

}  // namespace

extern "C" {

int cb_decoder_create(const cb_model* m, uint32_t max_step_tokens, uint32_t flags, cb_decoder** out) {
    return cb_decoder_create_batch(m, max_step_tokens, 1u, flags, out);
}

int cb_decoder_create_batch(const cb_model* m, uint32_t max_step_tokens, uint32_t sequences, uint32_t flags,
                            cb_decoder** out) {
    if (!m || !out || !m->layer) return fail(CB_ERROR_INVALID, "cb_decoder_create: null argument");
    if (sequences == 0 || sequences > 1024) return fail(CB_ERROR_INVALID, "cb_decoder_create: %u sequences", sequences);
    *out = nullptr;
    if (m->layers == 0 || m->hidden == 0 || m->hidden % 32 != 0 || m->hidden > 4096)
        return fail(CB_ERROR_BUILD, "cb_decoder_create: hidden width %u", m->hidden);
    if (m->head_dim != 64 && m->head_dim != 128 && m->head_dim != 256)
        return fail(CB_ERROR_BUILD, "cb_decoder_create: head dimension %u is not 64, 128 or 256", m->head_dim);
    if (m->kv_heads == 0 || m->query_heads % m->kv_heads != 0)
        return fail(CB_ERROR_BUILD, "cb_decoder_create: %u query heads do not share %u kv heads evenly",
                    m->query_heads, m->kv_heads);
    if (m->vocab < 64) return fail(CB_ERROR_BUILD, "cb_decoder_create: a vocabulary under the 64 candidates");
    if (m->context == 0 || max_step_tokens == 0 || max_step_tokens > 4096)
        return fail(CB_ERROR_BUILD, "cb_decoder_create: context %u, step tokens %u", m->context, max_step_tokens);
    cb_decoder* d = new (std::nothrow) cb_decoder();
    if (!d) return fail(CB_ERROR_BUILD, "cb_decoder_create: out of host memory");
    d->model = *m;
    d->max_tokens = max_step_tokens;
    d->sequences = sequences;
    d->rows = std::max(max_step_tokens, sequences);
    d->seq_next.assign(sequences, 0u);
    d->seq_drawn.assign(sequences, 0u);
    d->sms = sm_count();
    auto bail = [&](int rc) { cb_decoder_destroy(d); return rc; };
    if (d->sms <= 0) return bail(fail(CB_ERROR_BUILD, "cb_decoder_create: no CUDA device"));
    cudaError_t e = cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) return bail(fail_cuda(e, "cb_decoder_create: stream"));
    const uint32_t H = m->hidden, dh = m->head_dim, T = d->rows, S = sequences;
    if (int rc = upload_weight(d, &d->token_embd, m->token_embd, "token_embd")) return bail(rc);
    if (int rc = upload_weight(d, &d->output, m->output, "output")) return bail(rc);
    if (int rc = upload_f32(d, &d->output_norm, m->output_norm, H)) return bail(rc);
    if (int rc = upload_f32(d, &d->factors, m->rope_factors, dh / 2)) return bail(rc);
    d->layers.resize(m->layers);
    for (uint32_t l = 0; l < m->layers; ++l) {
        const cb_layer_weights& s = m->layer[l];
        DevLayer& L = d->layers[l];
        const char* names[7] = {"q", "k", "v", "o", "gate", "up", "down"};
        const cb_weight* srcs[7] = {&s.q, &s.k, &s.v, &s.o, &s.gate, &s.up, &s.down};
        DevWeight* dsts[7] = {&L.q, &L.k, &L.v, &L.o, &L.gate, &L.up, &L.down};
        for (int i = 0; i < 7; ++i) {
            if (srcs[i]->rows == 0) return bail(fail(CB_ERROR_BUILD, "cb_decoder_create: layer %u has no %s", l, names[i]));
            if (int rc = upload_weight(d, dsts[i], *srcs[i], names[i])) return bail(rc);
        }
        if (L.q.format != L.k.format || L.q.format != L.v.format || L.gate.format != L.up.format)
            return bail(fail(CB_ERROR_BUILD, "cb_decoder_create: layer %u's fused members differ in format", l));
        if (int rc = upload_f32(d, &L.attn_norm, s.attn_norm, H)) return bail(rc);
        if (int rc = upload_f32(d, &L.ffn_norm, s.ffn_norm, H)) return bail(rc);
        if (int rc = upload_f32(d, &L.post_attn_norm, s.post_attn_norm, H)) return bail(rc);
        if (int rc = upload_f32(d, &L.post_ffn_norm, s.post_ffn_norm, H)) return bail(rc);
        if (int rc = upload_f32(d, &L.q_norm, s.q_norm, dh)) return bail(rc);
        if (int rc = upload_f32(d, &L.k_norm, s.k_norm, dh)) return bail(rc);
        if (!L.attn_norm || !L.ffn_norm) return bail(fail(CB_ERROR_BUILD, "cb_decoder_create: layer %u norms", l));
        std::vector<float> turns(dh / 2);
        cb_rope_turns(s.rope_base, dh, turns.data());
        if (int rc = upload_f32(d, &L.turns, turns.data(), dh / 2)) return bail(rc);
        L.window = s.window ? s.window : m->context;
        // A sliding-window layer keeps a ring of its window and a step
        // (kv.h:13-34); a global layer the whole context.
        const uint64_t ring = static_cast<uint64_t>(L.window) + T;
        L.slots = static_cast<uint32_t>(L.window < m->context && ring < m->context ? ring : m->context);
        L.sequence_stride = static_cast<uint64_t>(L.slots) * m->kv_heads * dh;
        const size_t cache = static_cast<size_t>(L.sequence_stride) * S;
        if (int rc = dalloc(d, &L.key_cache, cache)) return bail(rc);
        if (int rc = dalloc(d, &L.value_cache, cache)) return bail(rc);
    }
    d->max_chunks = (m->context + 63u) / 64u;
    const size_t qd = static_cast<size_t>(m->query_heads) * dh, kvd = static_cast<size_t>(m->kv_heads) * dh;
    if (int rc = dalloc(d, &d->hidden, static_cast<size_t>(T) * H)) return bail(rc);
    if (int rc = dalloc(d, &d->normed, static_cast<size_t>(T) * H)) return bail(rc);
    if (int rc = dalloc(d, &d->hidden2, static_cast<size_t>(T) * H)) return bail(rc);
    if (int rc = dalloc(d, &d->q, T * qd)) return bail(rc);
    if (int rc = dalloc(d, &d->k, T * kvd)) return bail(rc);
    if (int rc = dalloc(d, &d->v, T * kvd)) return bail(rc);
    if (int rc = dalloc(d, &d->att, T * qd)) return bail(rc);
    if (int rc = dalloc(d, &d->out, static_cast<size_t>(T) * H)) return bail(rc);
    if (int rc = dalloc(d, &d->act, static_cast<size_t>(T) * m->ffn)) return bail(rc);
    if (int rc = dalloc(d, &d->logits, static_cast<size_t>(S) * m->vocab)) return bail(rc);
    if (int rc = dalloc(d, &d->partials, static_cast<size_t>(d->max_chunks) * T * qd)) return bail(rc);
    if (int rc = dalloc(d, &d->stats, static_cast<size_t>(d->max_chunks) * T * m->query_heads * 2)) return bail(rc);
    const uint32_t tickets = std::max(cb_attention_tickets(T, m->query_heads, m->kv_heads), S * m->kv_heads);
    if (int rc = dalloc(d, &d->tickets, tickets)) return bail(rc);
    if (int rc = dalloc(d, &d->sel_partials, static_cast<size_t>(S) * select_tiles(m->vocab) * 128)) return bail(rc);
    if (int rc = dalloc(d, &d->sel_ticket, static_cast<size_t>(S) * cb_select_tickets(m->vocab))) return bail(rc);
    if (int rc = dalloc(d, &d->candidates, static_cast<size_t>(S) * 128)) return bail(rc);
    if (int rc = dalloc(d, &d->sampled, static_cast<size_t>(S) * 4)) return bail(rc);
    if (int rc = dalloc(d, &d->ids, T)) return bail(rc);
    if (int rc = dalloc(d, &d->state, 2)) return bail(rc);
    if (flags & ~static_cast<uint32_t>(CB_DECODER_TENSOR_PREFILL))
        return bail(fail(CB_ERROR_INVALID, "cb_decoder_create: unknown flags 0x%x", flags));
    {
        // The split form's range sums for the widest product it may take:
        // non-gated products over K of 64 groups or more (o, down; QKV when
        // the hidden width is that wide).
        uint32_t rows = 0;
        if (qd / 32 >= 64 || m->ffn / 32 >= 64) rows = H;
        if (H / 32 >= 64) rows = std::max<uint32_t>(rows, static_cast<uint32_t>(qd + 2 * kvd));
        if (rows) {
            d->split_scratch_bytes = cb_matmul_split_bytes(T, rows);
            uint8_t* p = nullptr;
            if (int rc = dalloc(d, &p, d->split_scratch_bytes)) return bail(rc);
            d->split_scratch = p;
        }
    }
    if (flags & CB_DECODER_TENSOR_PREFILL) {
        // x16 for the widest K, then room for the dense form's split-K
        // partials of the non-gated products (up to 8 splits).
        const uint32_t widest = std::max<uint32_t>(std::max<uint32_t>(H, static_cast<uint32_t>(qd)), m->ffn);
        const uint64_t slots = std::max<uint64_t>(H, static_cast<uint64_t>(qd) + 2ull * kvd);
        d->tensor_scratch_bytes = cb_matmul_scratch_bytes(CB_MATMUL_TENSOR, T, widest) + 8ull * T * slots * 4ull;
        uint8_t* p = nullptr;
        if (int rc = dalloc(d, &p, d->tensor_scratch_bytes)) return bail(rc);
        d->tensor_scratch = p;
        d->tensor_prefill = true;
        uint16_t* h16 = nullptr;
        if (int rc = dalloc(d, &h16, static_cast<size_t>(T) * H)) return bail(rc);
        d->normed16 = h16;
        if (int rc = dalloc(d, &h16, static_cast<size_t>(T) * qd)) return bail(rc);
        d->att16 = h16;
        if (int rc = dalloc(d, &h16, static_cast<size_t>(T) * m->ffn)) return bail(rc);
        d->act16 = h16;
        // Every layer product's weights densified once.
        for (DevLayer& L : d->layers) {
            struct Want {
                cb_matmul m;
                void** dst;
            } wants[4] = {{description(d, {&L.q, &L.k, &L.v}, CB_EPILOGUE_QKV), &L.dense_qkv},
                          {description(d, {&L.o}, CB_EPILOGUE_WRITE), &L.dense_o},
                          {description(d, {&L.gate, &L.up}, CB_EPILOGUE_GATED), &L.dense_gate_up},
                          {description(d, {&L.down}, CB_EPILOGUE_WRITE), &L.dense_down}};
            for (Want& w : wants) {
                const uint64_t bytes = cb_matmul_dense_bytes(&w.m);
                if (bytes == 0) return bail(CB_ERROR_BUILD);
                uint8_t* q = nullptr;
                if (int rc = dalloc(d, &q, bytes)) return bail(rc);
                if (int rc = cb_matmul_densify(&w.m, q, bytes, d->stream)) return bail(rc);
                *w.dst = q;
            }
        }
        if (cudaError_t se = cudaStreamSynchronize(d->stream); se != cudaSuccess)
            return bail(fail_cuda(se, "cb_decoder_create: densify"));
    }
    e = cudaMemset(d->tickets, 0, tickets * sizeof(unsigned int));
    if (e == cudaSuccess)
        e = cudaMemset(d->sel_ticket, 0, static_cast<size_t>(S) * cb_select_tickets(m->vocab) * sizeof(unsigned int));
    if (e == cudaSuccess) e = cudaMemset(d->state, 0, 2 * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMemset(d->sampled, 0, static_cast<size_t>(S) * 4 * sizeof(uint32_t));
    if (e != cudaSuccess) return bail(fail_cuda(e, "cb_decoder_create: memset"));
    *out = d;
    return CB_OK;
}

void cb_decoder_destroy(cb_decoder* d) {
    if (!d) return;
    if (d->stream) cudaStreamSynchronize(d->stream);
    if (d->decode_graph) cudaGraphExecDestroy(d->decode_graph);
    if (d->step_graph) cudaGraphExecDestroy(d->step_graph);
    for (void* p : d->allocations) cudaFree(p);
    if (d->stream) cudaStreamDestroy(d->stream);
    delete d;
}

int cb_decoder_step(cb_decoder* d, const uint32_t* ids_host, uint32_t tokens, uint32_t position, uint32_t logits,
                    const cb_sampling* s, uint32_t* record_host) {
    return cb_decoder_step_sequence(d, 0, ids_host, tokens, position, logits, s, record_host);
}

int cb_decoder_step_sequence(cb_decoder* d, uint32_t seq, const uint32_t* ids_host, uint32_t tokens, uint32_t position,
                             uint32_t logits, const cb_sampling* s, uint32_t* record_host) {
    if (!d || !ids_host || tokens == 0) return fail(CB_ERROR_INVALID, "cb_decoder_step: null argument or no tokens");
    if (seq >= d->sequences) return fail(CB_ERROR_INVALID, "cb_decoder_step: sequence %u of %u", seq, d->sequences);
    if (tokens > d->max_tokens)
        return fail(CB_ERROR_INVALID, "cb_decoder_step: %u tokens over the step's %u", tokens, d->max_tokens);
    if (static_cast<uint64_t>(position) + tokens > d->model.context)
        return fail(CB_ERROR_STEP, "cb_decoder_step: positions past the context of %u", d->model.context);
    for (uint32_t i = 0; i < tokens; ++i)
        if (ids_host[i] >= d->model.vocab) return fail(CB_ERROR_INVALID, "cb_decoder_step: token %u", ids_host[i]);
    const cb_sampling greedy{0, 0, 1, 0.0f, 1.0f, 0.0f};
    const uint32_t st[2] = {position, 0};
    cudaError_t e = cudaMemcpyAsync(d->ids, ids_host, tokens * sizeof(uint32_t), cudaMemcpyHostToDevice, d->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d->state, st, sizeof st, cudaMemcpyHostToDevice, d->stream);
    if (e != cudaSuccess) return fail_cuda(e, "cb_decoder_step: upload");
    const cb_sampling smp = s ? *s : greedy;
    if (tokens == 1 && logits && d->sequences == 1) {
        // A decode step: the captured graph, replayed.
        if (d->step_graph && !same_sampling(smp, d->step_sampling)) {
            cudaGraphExecDestroy(d->step_graph);
            d->step_graph = nullptr;
        }
        if (!d->step_graph) {
            if (int rc = capture_step(d, false, smp, &d->step_graph)) return rc;
            d->step_sampling = smp;
        }
        e = cudaGraphLaunch(d->step_graph, d->stream);
        if (e != cudaSuccess) return fail_cuda(e, "cb_decoder_step: launch");
    } else if (int rc = enqueue_step(d, tokens, false, logits != 0, smp, static_cast<int>(seq))) {
        return rc;
    }
    if (logits && record_host) {
        e = cudaMemcpyAsync(record_host, d->sampled + 4u * seq, 4 * sizeof(uint32_t), cudaMemcpyDeviceToHost,
                            d->stream);
        if (e != cudaSuccess) return fail_cuda(e, "cb_decoder_step: readback");
    }
    e = cudaStreamSynchronize(d->stream);
    if (e != cudaSuccess) return fail_cuda(e, "cb_decoder_step");
    d->seq_drawn[seq] = logits != 0;
    d->seq_next[seq] = position + tokens;
    d->has_step = logits != 0;
    d->next_position = position + tokens;
    return finish_step(d);
}

int cb_decoder_step_batch(cb_decoder* d, const uint32_t* ids_host, uint32_t position, const cb_sampling* s,
                          uint32_t* records_host) {
    if (!d || !ids_host) return fail(CB_ERROR_INVALID, "cb_decoder_step_batch: null argument");
    const uint32_t S = d->sequences;
    if (static_cast<uint64_t>(position) + 1 > d->model.context)
        return fail(CB_ERROR_STEP, "cb_decoder_step_batch: position past the context of %u", d->model.context);
    for (uint32_t i = 0; i < S; ++i)
        if (ids_host[i] >= d->model.vocab) return fail(CB_ERROR_INVALID, "cb_decoder_step_batch: token %u", ids_host[i]);
    const cb_sampling greedy{0, 0, 1, 0.0f, 1.0f, 0.0f};
    const uint32_t st[2] = {position, 0};
    cudaError_t e = cudaMemcpyAsync(d->ids, ids_host, S * sizeof(uint32_t), cudaMemcpyHostToDevice, d->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d->state, st, sizeof st, cudaMemcpyHostToDevice, d->stream);
    if (e != cudaSuccess) return fail_cuda(e, "cb_decoder_step_batch: upload");
    if (int rc = enqueue_step(d, S, false, true, s ? *s : greedy, S > 1 ? -1 : 0)) return rc;
    if (records_host) {
        e = cudaMemcpyAsync(records_host, d->sampled, 4ull * S * sizeof(uint32_t), cudaMemcpyDeviceToHost, d->stream);
        if (e != cudaSuccess) return fail_cuda(e, "cb_decoder_step_batch: readback");
    }
    e = cudaStreamSynchronize(d->stream);
    if (e != cudaSuccess) return fail_cuda(e, "cb_decoder_step_batch");
    for (uint32_t i = 0; i < S; ++i) {
        d->seq_drawn[i] = 1;
        d->seq_next[i] = position + 1;
    }
    d->has_step = true;
    d->next_position = position + 1;
    return finish_step(d);
}

int cb_decoder_generate(cb_decoder* d, uint32_t steps, const cb_sampling* s, uint32_t* tokens_host,
                        uint32_t* failed_host, float* device_ms) {
    if (!d || !tokens_host) return fail(CB_ERROR_INVALID, "cb_decoder_generate: null argument");
    if (!d->has_step) return fail(CB_ERROR_INVALID, "cb_decoder_generate: no drawn token to feed");
    if (d->sequences > 1) {
        for (uint32_t i = 0; i < d->sequences; ++i)
            if (!d->seq_drawn[i] || d->seq_next[i] != d->seq_next[0])
                return fail(CB_ERROR_INVALID,
                            "cb_decoder_generate: every sequence needs a drawn token at one common position");
        d->next_position = d->seq_next[0];
    }
    if (steps == 0) return CB_OK;
    const cb_sampling greedy{0, 0, 1, 0.0f, 1.0f, 0.0f};
    const cb_sampling smp = s ? *s : greedy;
    cudaError_t e;
    if (steps > d->gen_capacity) {
        const uint32_t cap = steps < 4096 ? 4096 : steps;
        if (int rc = dalloc(d, &d->gen_tokens, static_cast<size_t>(cap) * d->sequences)) return rc;
        if (int rc = dalloc(d, &d->gen_failed, static_cast<size_t>(cap) * d->sequences)) return rc;
        d->gen_capacity = cap;
        if (d->decode_graph) { cudaGraphExecDestroy(d->decode_graph); d->decode_graph = nullptr; }
    }
    if (d->decode_graph && !same_sampling(smp, d->graph_sampling)) {
        cudaGraphExecDestroy(d->decode_graph);
        d->decode_graph = nullptr;
    }
    if (static_cast<uint64_t>(d->next_position) + steps > d->model.context)
        return fail(CB_ERROR_STEP, "cb_decoder_generate: positions past the context of %u", d->model.context);
    if (!d->decode_graph) {
        if (int rc = capture_step(d, true, smp, &d->decode_graph)) return rc;
        d->graph_sampling = smp;
    }
    // Fed steps start after the last step's tokens; the closing launch of
    // each advances the position and counts the step.
    const uint32_t st[2] = {d->next_position, 0};
    e = cudaMemcpyAsync(d->state, st, sizeof st, cudaMemcpyHostToDevice, d->stream);
    if (e != cudaSuccess) return fail_cuda(e, "cb_decoder_generate: state");
    cudaEvent_t ev[2] = {nullptr, nullptr};
    if (device_ms) {
        for (auto& x : ev)
            if ((e = cudaEventCreate(&x)) != cudaSuccess) return fail_cuda(e, "cb_decoder_generate: event");
        cudaEventRecord(ev[0], d->stream);
    }
    for (uint32_t i = 0; i < steps; ++i) {
        e = cudaGraphLaunch(d->decode_graph, d->stream);
        if (e != cudaSuccess) return fail_cuda(e, "cb_decoder_generate: launch");
    }
    if (device_ms) cudaEventRecord(ev[1], d->stream);
    const size_t n = static_cast<size_t>(steps) * d->sequences;
    e = cudaMemcpyAsync(tokens_host, d->gen_tokens, n * sizeof(uint32_t), cudaMemcpyDeviceToHost, d->stream);
    if (e == cudaSuccess && failed_host)
        e = cudaMemcpyAsync(failed_host, d->gen_failed, n * sizeof(uint32_t), cudaMemcpyDeviceToHost, d->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(d->stream);
    if (device_ms) {
        if (e == cudaSuccess) e = cudaEventElapsedTime(device_ms, ev[0], ev[1]);
        cudaEventDestroy(ev[0]);
        cudaEventDestroy(ev[1]);
    }
    if (e != cudaSuccess) return fail_cuda(e, "cb_decoder_generate");
    d->next_position += steps;
    for (auto& p : d->seq_next) p = d->next_position;
    return finish_step(d);
}

int cb_decoder_step_body(cb_decoder* d, const uint32_t* ids_host, uint32_t position) {
    if (!d) return fail(CB_ERROR_INVALID, "cb_decoder_step_body: null decoder");
    const uint32_t S = d->sequences;
    if (static_cast<uint64_t>(position) + 1 > d->model.context)
        return fail(CB_ERROR_STEP, "cb_decoder_step_body: position past the context of %u", d->model.context);
    const uint32_t st[2] = {position, 0};
    cudaError_t e = cudaSuccess;
    if (ids_host) {
        for (uint32_t i = 0; i < S; ++i)
            if (ids_host[i] >= d->model.vocab) return fail(CB_ERROR_INVALID, "cb_decoder_step_body: token %u", ids_host[i]);
        e = cudaMemcpyAsync(d->ids, ids_host, S * sizeof(uint32_t), cudaMemcpyHostToDevice, d->stream);
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(d->state, st, sizeof st, cudaMemcpyHostToDevice, d->stream);
    if (e != cudaSuccess) return fail_cuda(e, "cb_decoder_step_body: upload");
    const cb_sampling greedy{0, 0, 1, 0.0f, 1.0f, 0.0f};
    if (int rc = enqueue_step(d, S, ids_host == nullptr, true, greedy, S > 1 ? -1 : 0, false)) return rc;
    // the state copy's host array must outlive the copy
    e = cudaStreamSynchronize(d->stream);
    if (e != cudaSuccess) return fail_cuda(e, "cb_decoder_step_body");
    for (uint32_t i = 0; i < S; ++i) d->seq_next[i] = position + 1;
    d->next_position = position + 1;
    return CB_OK;
}

void* cb_decoder_stream(cb_decoder* d) { return d ? static_cast<void*>(d->stream) : nullptr; }
const float* cb_decoder_device_normed(cb_decoder* d) { return d ? d->normed : nullptr; }
uint32_t* cb_decoder_device_sampled(cb_decoder* d) { return d ? d->sampled : nullptr; }

int cb_decoder_head(cb_decoder* d, cb_member* head, uint32_t* format, uint32_t* columns) {
    if (!d || !head || !format || !columns) return fail(CB_ERROR_INVALID, "cb_decoder_head: null argument");
    const DevWeight& w = d->output.piece ? d->output : d->token_embd;
    *head = {w.piece, w.blocks, 0, w.rows, 0};
    *format = w.format;
    *columns = w.cols;
    return CB_OK;
}

int cb_decoder_logits_row(cb_decoder* d, uint32_t row, float* logits_host) {
    if (!d || !logits_host || row >= d->sequences) return fail(CB_ERROR_INVALID, "cb_decoder_logits_row: argument");
    const cudaError_t e = cudaMemcpy(logits_host, d->logits + static_cast<size_t>(row) * d->model.vocab,
                                     d->model.vocab * sizeof(float), cudaMemcpyDeviceToHost);
    return e == cudaSuccess ? CB_OK : fail_cuda(e, "cb_decoder_logits_row");
}

int cb_decoder_logits(cb_decoder* d, float* logits_host) {
    if (!d || !logits_host) return fail(CB_ERROR_INVALID, "cb_decoder_logits: null argument");
    const cudaError_t e = cudaMemcpy(logits_host, d->logits, d->model.vocab * sizeof(float), cudaMemcpyDeviceToHost);
    return e == cudaSuccess ? CB_OK : fail_cuda(e, "cb_decoder_logits");
}

const float* cb_decoder_device_logits(cb_decoder* d) { return d ? d->logits : nullptr; }

}  // extern "C"
