// C ABI entry points of the norm, rope, attention, gather and select
// kernels: argument checks (the reference launchers' preconditions), then
// the launch. A bad argument is CB_ERROR_INVALID before anything runs.
#include <cuda_runtime.h>

#include <cmath>

#include "api_common.h"
#include "charlotte_b200.h"
#include "formats.cuh"
#include "kernels.h"

using namespace cb;

namespace {

int launched(cudaError_t e, const char* what) { return e == cudaSuccess ? CB_OK : fail_cuda(e, what); }

bool head_dim_ok(uint32_t d) { return d == 64 || d == 128 || d == 256; }

}  // namespace

namespace cb {

int select_arguments(const cb_select* s, const char* who, bool own_scratch) {
    if (!s || !s->logits || !s->candidates || (!s->sampled && !s->candidates_only))
        return fail(CB_ERROR_INVALID, "%s: null argument", who);
    if (!own_scratch && (!s->partials || !s->ticket)) return fail(CB_ERROR_INVALID, "%s: null argument", who);
    if (s->rows > 1 && s->logits_stride < s->count)
        return fail(CB_ERROR_INVALID, "%s: rows overlap (logits_stride below count)", who);
    if (static_cast<uint64_t>(s->id_offset) + s->count > 0xFFFFFFFFull)
        return fail(CB_ERROR_INVALID, "%s: ids past 2^32 - 1", who);
    if (s->count == 0 || s->count > 262144) return fail(CB_ERROR_INVALID, "%s: %u entries (1 to 262,144)", who, s->count);
    return CB_OK;
}

}  // namespace cb

extern "C" {

int cb_norm_run(const cb_norm* n, uint32_t flags, void* stream) {
    if (!n || !n->hidden || (!n->normed && !n->add_only)) return fail(CB_ERROR_INVALID, "cb_norm_run: null argument");
    if ((n->scale || n->add_only) && !n->add)
        return fail(CB_ERROR_INVALID, "cb_norm_run: a scale or an add alone needs the add");
    if (n->rows_per_token > 1 && n->last_token)
        return fail(CB_ERROR_INVALID, "cb_norm_run: several rows a token with the last token's norm");
    if (n->width == 0 || n->width % 4 != 0 || n->width > 4096)
        return fail(CB_ERROR_INVALID, "cb_norm_run: width %u is not a multiple of 4 up to 4096", n->width);
    if (n->add && !n->output) return fail(CB_ERROR_INVALID, "cb_norm_run: add without the block's output");
    if (n->post_gain && !n->add) return fail(CB_ERROR_INVALID, "cb_norm_run: a post-norm needs the add");
    if (n->tokens == 0) return CB_OK;
    return launched(norm_run(*n, static_cast<cudaStream_t>(stream), flags & CB_RUN_PDL), "cb_norm_run");
}

void cb_rope_turns(double base, uint32_t head_dim, float* turns) {
    for (uint32_t k = 0; k < head_dim / 2; ++k) {
        const double theta = std::pow(base, -2.0 * k / head_dim);
        turns[k] = static_cast<float>(theta / (2 * 3.14159265358979323846));
    }
}

int cb_rope_run(const cb_rope* r, uint32_t flags, void* stream) {
    if (!r || !r->query || !r->key || !r->value || !r->turns || (!r->encode && (!r->key_cache || !r->value_cache)))
        return fail(CB_ERROR_INVALID, "cb_rope_run: null argument");
    if (r->encode && r->rows_are_sequences)
        return fail(CB_ERROR_INVALID, "cb_rope_run: the encode form takes the rows of one step");
    if (r->value_norm && !r->encode) return fail(CB_ERROR_INVALID, "cb_rope_run: value_norm is the encode form's");
    if (!head_dim_ok(r->head_dim) && !(r->encode && r->head_dim == 512))
        return fail(CB_ERROR_INVALID, "cb_rope_run: head dimension %u", r->head_dim);
    if (r->kv_heads == 0 || r->query_heads % r->kv_heads != 0)
        return fail(CB_ERROR_INVALID, "cb_rope_run: %u query heads over %u kv heads", r->query_heads, r->kv_heads);
    if ((r->query_heads + 2 * r->kv_heads) * (r->head_dim / 8) % 32 != 0)
        return fail(CB_ERROR_INVALID, "cb_rope_run: (Hq + 2 Hkv) * d / 8 is not a multiple of 32");
    if ((r->query_heads + 2 * r->kv_heads) * (r->head_dim / 8) > 1024)
        return fail(CB_ERROR_INVALID, "cb_rope_run: more than 1024 lanes a token");
    if ((r->query_gain == nullptr) != (r->key_gain == nullptr))
        return fail(CB_ERROR_INVALID, "cb_rope_run: QK-norm on queries or keys alone");
    if (r->slots == 0 && !r->encode) return fail(CB_ERROR_INVALID, "cb_rope_run: no cache slots");
    if (r->rows_are_sequences && r->sequence_stride < static_cast<uint64_t>(r->slots) * r->kv_heads * r->head_dim)
        return fail(CB_ERROR_INVALID, "cb_rope_run: sequences' caches overlap (stride below one cache)");
    if (r->tokens == 0) return CB_OK;
    return launched(rope_run(*r, static_cast<cudaStream_t>(stream), flags & CB_RUN_PDL), "cb_rope_run");
}

int cb_block_attention_run(const cb_block_attention* a, uint32_t flags, void* stream) {
    if (!a || !a->query || !a->key || !a->value || !a->out)
        return fail(CB_ERROR_INVALID, "cb_block_attention_run: null argument");
    if (a->head_dim == 0 || a->head_dim % 64 != 0 || a->head_dim > 512)
        return fail(CB_ERROR_INVALID, "cb_block_attention_run: head dimension %u", a->head_dim);
    if (a->kv_heads == 0 || a->query_heads % a->kv_heads != 0 || 16 % (a->query_heads / a->kv_heads) != 0)
        return fail(CB_ERROR_INVALID, "cb_block_attention_run: %u query heads over %u kv heads", a->query_heads,
                    a->kv_heads);
    if (!aligned16(a->query) || !aligned16(a->key) || !aligned16(a->value) || !aligned16(a->out))
        return fail(CB_ERROR_INVALID, "cb_block_attention_run: rows must be 16-byte aligned");
    if (a->tokens == 0) return CB_OK;
    if (!block_attention_fits(*a))
        return fail(CB_ERROR_INVALID, "cb_block_attention_run: %u tokens of head dimension %u do not fit", a->tokens,
                    a->head_dim);
    return launched(block_attention_run(*a, static_cast<cudaStream_t>(stream), flags & CB_RUN_PDL),
                    "cb_block_attention_run");
}

int cb_pool_run(const cb_pool* p, uint32_t flags, void* stream) {
    if (!p || !p->input || !p->output) return fail(CB_ERROR_INVALID, "cb_pool_run: null argument");
    if (p->kind != CB_POOL_MEAN && p->kind != CB_POOL_UNIT) return fail(CB_ERROR_INVALID, "cb_pool_run: kind %u", p->kind);
    if (p->width == 0 || p->width % 4 != 0 || p->width > 4096)
        return fail(CB_ERROR_INVALID, "cb_pool_run: width %u is not a multiple of 4 up to 4096", p->width);
    if (!aligned16(p->input) || !aligned16(p->output))
        return fail(CB_ERROR_INVALID, "cb_pool_run: rows must be 16-byte aligned");
    if (p->tokens == 0) return CB_OK;
    return launched(pool_run(*p, static_cast<cudaStream_t>(stream), flags & CB_RUN_PDL), "cb_pool_run");
}

uint32_t cb_attention_tickets(uint32_t tokens, uint32_t query_heads, uint32_t kv_heads) {
    if (kv_heads == 0) return 0;
    return attention_row_tiles(tokens, query_heads, kv_heads, false) * kv_heads;
}

int cb_attention_run(const cb_attention* a, uint32_t flags, void* stream) {
    if (!a || !a->query || !a->key_cache || !a->value_cache || !a->out || !a->partials || !a->stats || !a->tickets)
        return fail(CB_ERROR_INVALID, "cb_attention_run: null argument");
    if (!head_dim_ok(a->head_dim)) return fail(CB_ERROR_INVALID, "cb_attention_run: head dimension %u", a->head_dim);
    if (a->kv_heads == 0 || a->query_heads % a->kv_heads != 0 || a->query_heads / a->kv_heads > 16)
        return fail(CB_ERROR_INVALID, "cb_attention_run: %u query heads over %u kv heads", a->query_heads,
                    a->kv_heads);
    if (a->slots == 0 || a->window == 0) return fail(CB_ERROR_INVALID, "cb_attention_run: no slots or no window");
    if (!aligned16(a->key_cache) || !aligned16(a->value_cache) || !aligned16(a->query))
        return fail(CB_ERROR_INVALID, "cb_attention_run: caches and queries must be 16-byte aligned");
    if (a->rows_are_sequences && a->sequence_stride < static_cast<uint64_t>(a->slots) * a->kv_heads * a->head_dim)
        return fail(CB_ERROR_INVALID, "cb_attention_run: sequences' caches overlap (stride below one cache)");
    if (!a->position && static_cast<uint64_t>(a->position0) + (a->rows_are_sequences ? 1u : a->tokens) >
                            static_cast<uint64_t>(a->max_chunks) * 64)
        return fail(CB_ERROR_INVALID, "cb_attention_run: positions past max_chunks");
    if (const cb_rope* r = a->rope) {
        if (!(a->tokens == 1 || a->rows_are_sequences))
            return fail(CB_ERROR_INVALID, "cb_attention_run: a fused rope needs a decode shape (one token, or sequences)");
        if (!r->query || !r->key || !r->value || !r->turns || !aligned16(r->query) || !aligned16(r->key) ||
            !aligned16(r->value))
            return fail(CB_ERROR_INVALID, "cb_attention_run: fused rope: null or unaligned rows");
        if (r->tokens != a->tokens || r->head_dim != a->head_dim || r->query_heads != a->query_heads ||
            r->kv_heads != a->kv_heads || r->slots != a->slots || r->key_cache != a->key_cache ||
            r->value_cache != a->value_cache || r->position != a->position ||
            (!a->position && r->position0 != a->position0) ||
            (r->rows_are_sequences != 0) != (a->rows_are_sequences != 0) ||
            (a->rows_are_sequences && r->sequence_stride != a->sequence_stride))
            return fail(CB_ERROR_INVALID, "cb_attention_run: the fused rope describes other rows, heads or caches");
        if ((r->query_gain == nullptr) != (r->key_gain == nullptr))
            return fail(CB_ERROR_INVALID, "cb_attention_run: fused rope: both norm gains or neither");
    }
    if (a->tokens == 0) return CB_OK;
    if ((flags & CB_RUN_TENSOR) && !a->rope && attention_tensor_fits(*a))
        return launched(attention_tensor_run(*a, static_cast<cudaStream_t>(stream), flags & CB_RUN_PDL),
                        "cb_attention_run");
    return launched(attention_run(*a, static_cast<cudaStream_t>(stream), flags & CB_RUN_PDL), "cb_attention_run");
}

int cb_gather_run(const cb_gather* g, uint32_t flags, void* stream) {
    if (!g || !g->piece || !g->hidden || (!g->fed && !g->ids) || (g->fed && !g->sampled))
        return fail(CB_ERROR_INVALID, "cb_gather_run: null argument");
    if (g->format != CB_Q4_0 && g->format != CB_Q4_1 && g->format != CB_Q8_0 && g->format != CB_Q6_K &&
        g->format != CB_BF16)
        return fail(CB_ERROR_INVALID, "cb_gather_run: format %u", g->format);
    if (g->width == 0 || g->width % (g->format == CB_Q6_K ? 256 : 32) != 0)
        return fail(CB_ERROR_INVALID, "cb_gather_run: width %u is not whole blocks", g->width);
    if (g->fed && g->tokens != 1 && g->fed_stride == 0)
        return fail(CB_ERROR_INVALID, "cb_gather_run: a fed step of several rows needs fed_stride");
    if (g->tokens == 0) return CB_OK;
    return launched(gather_run(*g, static_cast<cudaStream_t>(stream), flags & CB_RUN_PDL), "cb_gather_run");
}

uint32_t cb_select_tiles(uint32_t count) { return select_tiles(count); }

uint32_t cb_select_tickets(uint32_t count) { return 1u + (select_tiles(count) + 15u) / 16u; }

int cb_select_run(const cb_select* s, uint32_t flags, void* stream) {
    if (int rc = select_arguments(s, "cb_select_run", false)) return rc;
    return launched(select_run(*s, static_cast<cudaStream_t>(stream), flags & CB_RUN_PDL), "cb_select_run");
}

int cb_select_merge_run(const cb_select_merge* m, uint32_t flags, void* stream) {
    if (!m || !m->lists_data || !m->candidates || !m->sampled)
        return fail(CB_ERROR_INVALID, "cb_select_merge_run: null argument");
    if (m->lists == 0 || m->lists > 64) return fail(CB_ERROR_INVALID, "cb_select_merge_run: %u lists (1 to 64)", m->lists);
    if (m->rows == 0) return CB_OK;
    return launched(select_merge_run(*m, static_cast<cudaStream_t>(stream), flags & CB_RUN_PDL), "cb_select_merge_run");
}

}  // extern "C"
