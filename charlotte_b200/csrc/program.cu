// The reference's kernels::Program over CUDA (plainsight-systems/charlotte,
// src/core/kernels/program.h:262-331): a graph's launches, as the reference's
// launchers describe them (kernels::Launch, src/core/kernels/interface.h:
// 318-365, here cb_launch), built once onto this library's kernels and run a
// step at a time.
//
// Build: each launch's kernel, entry point, constants, bindings and
// overrides become one operation on the kernels behind the C ABI
// (cb_matmul_run, cb_norm_run, cb_rope_run, cb_attention_run, cb_gather_run,
// cb_select_run, cb_select_merge_run), with device pointers resolved from
// the plan's buffers. A few reference launches have no work of their own
// here: a split product's range-sum launches and its combine are one
// product, given the reference's range_sums buffer as the split form's
// scratch (every exact form adds the 32 ranges in order), attention's combine is
// part of its main launch, and the top-k passes are one selection, which
// also makes the draw that follows it. A launch this backend has no form for
// is refused at build, named.
//
// Run: the step's 64-byte head and its identifiers are copied to a device
// copy of the Step (the reference's binding 0), which the kernels read their
// position, identifiers and fed token from; then every operation the step
// runs (its token range, last-token launches only when it asks for logits:
// interface.h workgroups_for) in the graph's order on the program's stream,
// then the readback and the device's fault word into pinned host memory,
// and an event. A one-token step replays a CUDA graph captured once for its
// logits, fed and sampling settings. At most two steps are outstanding
// (program.h:62-70); cb_program_poll fires their callbacks in run order
// (kernels/order.h:30).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <deque>
#include <new>
#include <string>
#include <vector>

#include "api_common.h"
#include "charlotte_b200.h"
#include "kernels.h"

struct cb_buffers {
    std::vector<void*> ptr;
    std::vector<uint64_t> size;
};

namespace {

using namespace cb;

constexpr uint32_t kOutstanding = 2;           // program.h: one running, one queued
constexpr uint32_t kMaxPositions = 1u << 24;   // interface.h kMaxPositions
constexpr uint32_t kPrefillBlock = 512;        // residency kPrefillBlock: a step's most tokens
constexpr uint32_t kStepHead = 64;             // interface.h kStepHead
constexpr uint64_t kMaxReadback = 4096;        // program.h kMaxReadback
constexpr uint32_t kGgufF16 = 1;

enum class Kind { Matmul, Norm, Rope, Attention, Gather, Select, Draw, BlockAttention, Pool };

// One operation: the launches [first_launch, last_launch] of the graph.
struct Op {
    Kind kind = Kind::Matmul;
    uint32_t first_launch = 0, last_launch = 0;
    uint32_t least = 1, most = UINT32_MAX;   // the step token counts it runs in
    bool last_token = false;                  // runs only in steps that ask for logits
    // Matmul
    cb_matmul mm{};
    const float* x = nullptr;
    uint32_t x_stride = 0;
    float* out[3] = {nullptr, nullptr, nullptr};
    uint32_t out_stride[3] = {0, 0, 0};
    bool decode_form = false;   // one row: the step's only token, or its last
    // the other kernels' arguments, patched with the step's values at run
    cb_norm norm{};
    cb_rope rope{};
    cb_attention att{};
    cb_gather gather{};
    cb_select sel{};
    bool select_draws = false;
    cb_select_merge draw{};
    cb_block_attention block{};
    cb_pool pool{};
};

struct Graph {
    uint32_t logits = 0, fed = 0;
    uint32_t seed[2] = {0, 0}, top_k = 0;
    float temperature = 0, top_p = 0, min_p = 0, log_min_p = 0;
    cudaGraphExec_t exec = nullptr;
};

struct Pending {
    uint64_t number = 0;
    uint32_t slot = 0;
    int status = CB_OK;
    std::string message;
    bool reads_back = false;
    bool profiled = false;
    cb_step_callback done = nullptr;
    cb_profile_callback profile_done = nullptr;
    void* userdata = nullptr;
    std::vector<uint32_t> timed;   // launch index of each timed operation's end
};

struct Slot {
    cb_step* step_host = nullptr;       // pinned
    uint8_t* readback_host = nullptr;   // pinned
    unsigned int* fault_host = nullptr; // pinned
    cudaEvent_t done = nullptr;
    cudaEvent_t begin = nullptr;        // profiled steps
    std::vector<cudaEvent_t> marks;     // profiled steps: one after each operation
};

bool is(const char* a, const char* b) { return a && std::strcmp(a, b) == 0; }

bool starts(const char* a, const char* prefix) { return a && std::strncmp(a, prefix, std::strlen(prefix)) == 0; }

}  // namespace

struct cb_program {
    cb_buffers* buffers = nullptr;
    uint32_t launch_count = 0;
    std::vector<Op> ops;
    cudaStream_t stream = nullptr;
    cb_step* step_device = nullptr;
    std::vector<void*> owned;            // device memory of the program's own
    float* partials = nullptr;
    float* stats = nullptr;
    unsigned int* tickets = nullptr;
    uint32_t ticket_words = 0;
    uint32_t* sel_partials = nullptr;
    unsigned int* sel_ticket = nullptr;
    uint32_t sel_ticket_words = 0;
    uint32_t max_chunks = 0;
    const void* readback = nullptr;
    uint64_t readback_bytes = 0;
    Slot slots[kOutstanding];
    std::deque<Pending> pending;
    uint64_t next_number = 0;
    std::vector<Graph> graphs;
};

namespace {

int dev_alloc(cb_program* p, void** out, size_t bytes) {
    void* q = nullptr;
    const cudaError_t e = cudaMalloc(&q, bytes ? bytes : 16);
    if (e != cudaSuccess) return fail_cuda(e, "cb_program_build: cudaMalloc");
    p->owned.push_back(q);
    *out = q;
    return CB_OK;
}

// A binding's device address, checked against its buffer.
int resolve(const cb_program* p, const cb_binding& b, uint32_t index, void** out) {
    const cb_buffers* bufs = p->buffers;
    if (b.buffer >= bufs->ptr.size() || b.offset > bufs->size[b.buffer] || b.size > bufs->size[b.buffer] - b.offset)
        return fail(CB_ERROR_BUILD, "cb_program_build: launch %u binds outside buffer %u", index, b.buffer);
    *out = static_cast<uint8_t*>(bufs->ptr[b.buffer]) + b.offset;
    return CB_OK;
}

bool override_of(const cb_launch& l, const char* name, double* value) {
    for (uint32_t i = 0; i < l.override_count; ++i)
        if (is(l.overrides[i].name, name)) {
            *value = l.overrides[i].value;
            return true;
        }
    return false;
}

double override_or(const cb_launch& l, const char* name, double fallback) {
    double v = fallback;
    override_of(l, name, &v);
    return v;
}

template <typename T>
T constant_at(const cb_launch& l, uint32_t offset) {
    T v{};
    if (l.constants && offset + sizeof(T) <= l.constants_bytes) std::memcpy(&v, l.constants + offset, sizeof(T));
    return v;
}

void set_range(Op& op, const cb_launch& l, uint32_t index) {
    op.first_launch = op.last_launch = index;
    op.least = l.tokens_least ? l.tokens_least : 1u;
    op.most = l.tokens_most ? l.tokens_most : UINT32_MAX;
    op.last_token = l.rows == CB_ROWS_LAST_TOKEN;
}

// matmul.wgsl's Matmul constants (src/core/kernels/matmul/matmul.cpp:39-52):
// members[3] of {first word in the weights binding, blocks, first output row
// (a gated member: its first row within its weight), rows}, then
// gate_input {row stride, first column}, clip and bias words.
struct MatmulConstants {
    uint32_t member[3][4];
    uint32_t gate_input[4];
    uint32_t clip[4];
    uint32_t bias[4];
};

// A product launch (decode_*, prefill_*, or a split's combine_*) as one
// cb_matmul: `weights` and `input` are the product's own bindings (a
// combine takes them from its split launch), `outputs` its outputs then
// GatedByInput's u.
int build_matmul(cb_program* p, const cb_launch& l, uint32_t index, const char* epilogue_name, bool decode,
                 const cb_binding& weights, const cb_binding& input, const cb_binding* outputs, uint32_t output_count,
                 Op& op) {
    if (l.constants_bytes < sizeof(MatmulConstants))
        return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: matmul constants of %u bytes", index,
                    l.constants_bytes);
    for (const char* option : {"clipped", "biased", "activated"})
        if (override_or(l, option, 0.0) != 0.0)
            return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: the matmul option '%s' has no CUDA form", index,
                        option);
    MatmulConstants c{};
    std::memcpy(&c, l.constants, sizeof c);
    uint32_t epilogue;
    if (is(epilogue_name, "write")) epilogue = CB_EPILOGUE_WRITE;
    else if (is(epilogue_name, "qkv")) epilogue = CB_EPILOGUE_QKV;
    else if (is(epilogue_name, "gated")) epilogue = CB_EPILOGUE_GATED;
    else if (is(epilogue_name, "gated_input")) epilogue = CB_EPILOGUE_GATED_BY_INPUT;
    else return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: matmul entry point %s", index, l.entry_point);
    const uint32_t outputs_needed = (epilogue == CB_EPILOGUE_QKV ? 3u : 1u) + (epilogue == CB_EPILOGUE_GATED_BY_INPUT);
    if (output_count < outputs_needed)
        return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: %u output bindings for %s", index, output_count,
                    l.entry_point);
    void* wbase = nullptr;
    void* xin = nullptr;
    if (int rc = resolve(p, weights, index, &wbase)) return rc;
    if (int rc = resolve(p, input, index, &xin)) return rc;
    const uint32_t columns = static_cast<uint32_t>(override_or(l, "columns", 0.0));
    if (columns == 0) return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: no columns override", index);
    cb_matmul& m = op.mm;
    m = {};
    m.format = l.format;
    m.columns = columns;
    m.epilogue = epilogue;
    m.activation = static_cast<uint32_t>(override_or(l, "activation", 0.0));
    uint32_t members = 0;
    for (uint32_t i = 0; i < 3; ++i) {
        if (c.member[i][3] == 0) break;
        cb_member& mb = m.member[i];
        mb.piece = static_cast<uint8_t*>(wbase) + 4ull * c.member[i][0];
        mb.blocks = c.member[i][1];
        mb.rows = c.member[i][3];
        if (epilogue == CB_EPILOGUE_GATED) {
            mb.first_row = c.member[i][2];   // the member's first row within its weight
            mb.out_offset = 0;
        } else if (epilogue == CB_EPILOGUE_QKV) {
            mb.first_row = 0;                // member m's rows go to output m
            mb.out_offset = 0;
        } else {
            mb.first_row = 0;
            mb.out_offset = c.member[i][2];  // its first output row
        }
        ++members;
    }
    if (members == 0) return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: a product of no rows", index);
    m.members = members;
    op.kind = Kind::Matmul;
    op.x = static_cast<const float*>(xin);
    op.x_stride = columns;
    op.decode_form = decode;
    const uint32_t outs = epilogue == CB_EPILOGUE_QKV ? 3u : 1u;
    for (uint32_t o = 0; o < outs; ++o) {
        void* ptr = nullptr;
        if (int rc = resolve(p, outputs[o], index, &ptr)) return rc;
        op.out[o] = static_cast<float*>(ptr);
    }
    // Output row widths (matmul.wgsl:529-586): a Write's out_width, a QKV
    // member's rows, a gated product's gate rows.
    if (epilogue == CB_EPILOGUE_QKV) {
        for (uint32_t o = 0; o < 3; ++o) op.out_stride[o] = c.member[o][3];
    } else if (epilogue == CB_EPILOGUE_GATED) {
        op.out_stride[0] = c.member[0][3];
    } else {
        op.out_stride[0] = static_cast<uint32_t>(override_or(l, "out_width", 0.0));
    }
    if (epilogue == CB_EPILOGUE_GATED_BY_INPUT) {
        void* u = nullptr;
        if (int rc = resolve(p, outputs[1], index, &u)) return rc;
        m.gate_input = static_cast<const float*>(u);
        m.gate_input_stride = c.gate_input[0];
        m.gate_input_column = c.gate_input[1];
    }
    return CB_OK;
}

int build_one(cb_program* p, const cb_launch* launches, uint32_t count, uint32_t& i, std::vector<Op>& ops) {
    const cb_launch& l = launches[i];
    const char* entry = l.entry_point ? l.entry_point : "main";
    Op op{};
    set_range(op, l, i);
    switch (l.kernel) {
        case CB_KERNEL_MATMUL: {
            if (is(entry, "split_ranges")) {
                // Its combine (after this product's tile launches) is the product.
                return CB_OK;
            }
            const bool decode = starts(entry, "decode_");
            const bool prefill = starts(entry, "prefill_");
            const bool combine = starts(entry, "combine_");
            if (!decode && !prefill && !combine)
                return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: matmul entry point %s", i, entry);
            const char* epi = entry + (decode ? 7 : (prefill ? 8 : 8));
            if (combine) {
                // The split launch this combine closes: the nearest earlier
                // split_ranges of the same constants, whose bindings are
                // {weights, input, range sums}.
                const cb_launch* split = nullptr;
                for (uint32_t j = i; j-- > 0;) {
                    const cb_launch& s = launches[j];
                    if (s.kernel == CB_KERNEL_MATMUL && is(s.entry_point, "split_ranges") &&
                        s.constants_bytes == l.constants_bytes &&
                        std::memcmp(s.constants, l.constants, l.constants_bytes) == 0) {
                        split = &s;
                        break;
                    }
                }
                if (!split || split->binding_count < 3 || l.binding_count < 2)
                    return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: a combine without its split", i);
                if (int rc = build_matmul(p, l, i, epi, false, split->bindings[0], split->bindings[1], l.bindings + 1,
                                          l.binding_count - 1, op))
                    return rc;
                // The split's range sums (the reference's range_sums buffer,
                // in its layout) are the split form's scratch; the library
                // takes the split form where it pays (cb_matmul_run).
                void* sums = nullptr;
                if (int rc = resolve(p, split->bindings[2], i, &sums)) return rc;
                op.mm.scratch = sums;
                op.mm.scratch_bytes = split->bindings[2].size;
            } else {
                if (l.binding_count < 3)
                    return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: %u matmul bindings", i, l.binding_count);
                if (int rc = build_matmul(p, l, i, epi, decode, l.bindings[0], l.bindings[1], l.bindings + 2,
                                          l.binding_count - 2, op))
                    return rc;
            }
            ops.push_back(op);
            return CB_OK;
        }
        case CB_KERNEL_NORM: {
            if (!is(entry, "main")) return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: norm entry %s", i, entry);
            if (l.binding_count < 5) return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: norm bindings", i);
            // The audio encoder's forms (a re-norm, a post scale) have no CUDA form.
            if (override_or(l, "renorm", 0.0) != 0.0 || constant_at<float>(l, 4) != 1.0f)
                return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: a norm with a re-norm or a post scale has "
                            "no CUDA form", i);
            const bool scaled = override_or(l, "scaled", 0.0) != 0.0;
            if (scaled && l.binding_count < 6) return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: norm scale", i);
            void* ptr[6] = {};
            for (uint32_t b = 0; b < (scaled ? 6u : 5u); ++b)
                if (int rc = resolve(p, l.bindings[b], i, &ptr[b])) return rc;
            const bool add = override_or(l, "add", 0.0) != 0.0;
            const bool post = override_or(l, "post_norm", 0.0) != 0.0;
            const bool unit = override_or(l, "unit_gain", 0.0) != 0.0;
            cb_norm& n = op.norm;
            n.gain = unit ? nullptr : static_cast<const float*>(ptr[0]);
            n.post_gain = post ? static_cast<const float*>(ptr[1]) : nullptr;
            n.output = add ? static_cast<const float*>(ptr[2]) : nullptr;
            n.hidden = static_cast<float*>(ptr[3]);
            n.normed = static_cast<float*>(ptr[4]);
            n.width = static_cast<uint32_t>(override_or(l, "width", 0.0));
            n.add = add ? 1u : 0u;
            n.last_token = op.last_token ? 1u : 0u;
            n.epsilon = constant_at<float>(l, 0);
            n.scale = scaled ? static_cast<const float*>(ptr[5]) : nullptr;
            n.add_only = override_or(l, "normalize", 1.0) == 0.0 ? 1u : 0u;
            n.rows_per_token = static_cast<uint32_t>(override_or(l, "rows_per_token", 1.0));
            op.kind = Kind::Norm;
            ops.push_back(op);
            return CB_OK;
        }
        case CB_KERNEL_ROPE_CACHE: {
            if (!is(entry, "main")) return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: rope entry %s", i, entry);
            if (l.binding_count < 8) return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: rope bindings", i);
            if (override_or(l, "axial", 0.0) != 0.0 || override_or(l, "value_norm", 0.0) != 0.0)
                return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: the axial or value-normed rope has no CUDA "
                            "form", i);
            if (l.pack_format != kGgufF16)
                return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: a cache packed as type %u (F16 only)", i,
                            l.pack_format);
            void* ptr[8];
            for (uint32_t b = 0; b < 8; ++b)
                if (int rc = resolve(p, l.bindings[b], i, &ptr[b])) return rc;
            const uint32_t d = static_cast<uint32_t>(override_or(l, "head_dimension", 0.0));
            if (d == 0 || d > 512 || l.constants_bytes < 16 + 4 * (d / 2))
                return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: rope of head dimension %u", i, d);
            // the turns (rope.cpp:76-87), at offset 16 of the constants, to the device
            void* turns = nullptr;
            if (int rc = dev_alloc(p, &turns, 4 * (d / 2))) return rc;
            const cudaError_t e = cudaMemcpy(turns, l.constants + 16, 4 * (d / 2), cudaMemcpyHostToDevice);
            if (e != cudaSuccess) return fail_cuda(e, "cb_program_build: rope turns");
            const bool qk = override_or(l, "qk_norm", 0.0) != 0.0;
            const bool factors = override_or(l, "factors", 0.0) != 0.0;
            cb_rope& r = op.rope;
            r.query_gain = qk ? static_cast<const float*>(ptr[0]) : nullptr;
            r.key_gain = qk ? static_cast<const float*>(ptr[1]) : nullptr;
            r.factors = factors ? static_cast<const float*>(ptr[2]) : nullptr;
            r.query = static_cast<float*>(ptr[3]);
            r.key = static_cast<float*>(ptr[4]);
            r.value = static_cast<float*>(ptr[5]);
            r.key_cache = static_cast<uint16_t*>(ptr[6]);
            r.value_cache = static_cast<uint16_t*>(ptr[7]);
            r.turns = static_cast<const float*>(turns);
            r.head_dim = d;
            r.query_heads = static_cast<uint32_t>(override_or(l, "query_heads", 0.0));
            r.kv_heads = static_cast<uint32_t>(override_or(l, "key_value_heads", 0.0));
            r.halves = override_or(l, "halves", 0.0) != 0.0 ? 1u : 0u;
            r.slots = constant_at<uint32_t>(l, 0);
            r.epsilon = constant_at<float>(l, 4);
            op.kind = Kind::Rope;
            ops.push_back(op);
            return CB_OK;
        }
        case CB_KERNEL_ROPE_ENCODE: {
            // rope_encode_launch (rope.cpp): bindings {query gain, key gain,
            // factors, query, key, value}; constants {slots, ε, turns at 16}.
            if (!is(entry, "main")) return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: rope entry %s", i, entry);
            if (l.binding_count < 6) return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: rope bindings", i);
            const uint32_t d = static_cast<uint32_t>(override_or(l, "head_dimension", 0.0));
            if (override_or(l, "axial", 0.0) != 0.0 || (d != 64 && d != 128 && d != 256 && d != 512))
                return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: rope's encode form %s has no CUDA form", i,
                            override_or(l, "axial", 0.0) != 0.0 ? "in the axial pairing" : "at this head dimension");
            if (l.constants_bytes < 16 + 4 * (d / 2))
                return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: rope constants", i);
            void* ptr[6];
            for (uint32_t b = 0; b < 6; ++b)
                if (int rc = resolve(p, l.bindings[b], i, &ptr[b])) return rc;
            void* turns = nullptr;
            if (int rc = dev_alloc(p, &turns, 4 * (d / 2))) return rc;
            const cudaError_t e = cudaMemcpy(turns, l.constants + 16, 4 * (d / 2), cudaMemcpyHostToDevice);
            if (e != cudaSuccess) return fail_cuda(e, "cb_program_build: rope turns");
            const bool qk = override_or(l, "qk_norm", 0.0) != 0.0;
            const bool factors = override_or(l, "factors", 0.0) != 0.0;
            cb_rope& r = op.rope;
            r.query_gain = qk ? static_cast<const float*>(ptr[0]) : nullptr;
            r.key_gain = qk ? static_cast<const float*>(ptr[1]) : nullptr;
            r.factors = factors ? static_cast<const float*>(ptr[2]) : nullptr;
            r.query = static_cast<float*>(ptr[3]);
            r.key = static_cast<float*>(ptr[4]);
            r.value = static_cast<float*>(ptr[5]);
            r.turns = static_cast<const float*>(turns);
            r.head_dim = d;
            r.query_heads = static_cast<uint32_t>(override_or(l, "query_heads", 0.0));
            r.kv_heads = static_cast<uint32_t>(override_or(l, "key_value_heads", 0.0));
            r.halves = override_or(l, "halves", 0.0) != 0.0 ? 1u : 0u;
            r.epsilon = constant_at<float>(l, 4);
            r.encode = 1;
            r.value_norm = override_or(l, "value_norm", 0.0) != 0.0 ? 1u : 0u;
            op.kind = Kind::Rope;
            ops.push_back(op);
            return CB_OK;
        }
        case CB_KERNEL_BLOCK_ATTENTION: {
            // block_attention_launches (block_attention.cpp): scores_of
            // {query, key, scores, maxima} then weigh {scores, maxima, value,
            // attention}, one launch here; constants {half window, scale·log2e}.
            if (!is(entry, "scores_of"))
                return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: block attention entry %s without its scores",
                            i, entry);
            if (i + 1 >= count || launches[i + 1].kernel != CB_KERNEL_BLOCK_ATTENTION ||
                !is(launches[i + 1].entry_point, "weigh") || l.binding_count < 2 || launches[i + 1].binding_count < 4)
                return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: block attention's scores without its weigh", i);
            void* ptr[4];
            for (uint32_t b = 0; b < 2; ++b)
                if (int rc = resolve(p, l.bindings[b], i, &ptr[b])) return rc;
            for (uint32_t b = 2; b < 4; ++b)
                if (int rc = resolve(p, launches[i + 1].bindings[b], i + 1, &ptr[b])) return rc;
            cb_block_attention& a = op.block;
            a.query = static_cast<const float*>(ptr[0]);
            a.key = static_cast<const float*>(ptr[1]);
            a.value = static_cast<const float*>(ptr[2]);
            a.out = static_cast<float*>(ptr[3]);
            a.head_dim = static_cast<uint32_t>(override_or(l, "head_dimension", 0.0));
            a.query_heads = static_cast<uint32_t>(override_or(l, "query_heads", 0.0));
            a.kv_heads = static_cast<uint32_t>(override_or(l, "key_value_heads", 0.0));
            a.half_window = constant_at<uint32_t>(l, 0);
            a.scale_log2e = constant_at<float>(l, 4);
            if (a.kv_heads == 0 || a.query_heads % a.kv_heads != 0 || 16 % (a.query_heads / a.kv_heads) != 0 ||
                a.head_dim % 64 != 0 || a.head_dim > 512)
                return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: block attention of %u/%u heads of %u", i,
                            a.query_heads, a.kv_heads, a.head_dim);
            op.kind = Kind::BlockAttention;
            op.last_launch = i + 1;
            ops.push_back(op);
            i = i + 1;
            return CB_OK;
        }
        case CB_KERNEL_POOL: {
            // mean_launch / unit_launch (pool.cpp): {input, output};
            // constants {vec4s, pooling, ε}.
            const bool mean = is(entry, "mean");
            if (!mean && !is(entry, "unit"))
                return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: pooling entry %s has no CUDA form", i, entry);
            if (l.binding_count < 2) return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: pool bindings", i);
            void* ptr[2];
            for (uint32_t b = 0; b < 2; ++b)
                if (int rc = resolve(p, l.bindings[b], i, &ptr[b])) return rc;
            cb_pool& q = op.pool;
            q.input = static_cast<const float*>(ptr[0]);
            q.output = static_cast<float*>(ptr[1]);
            q.width = 4u * constant_at<uint32_t>(l, 0);
            q.kind = mean ? CB_POOL_MEAN : CB_POOL_UNIT;
            op.kind = Kind::Pool;
            ops.push_back(op);
            return CB_OK;
        }
        case CB_KERNEL_ATTENTION: {
            if (is(entry, "combine")) return CB_OK;   // folded by the main launch
            if (!is(entry, "main"))
                return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: attention entry %s", i, entry);
            if (l.binding_count < 4) return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: attention bindings", i);
            if (l.pack_format != kGgufF16)
                return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: a cache of type %u (F16 only)", i,
                            l.pack_format);
            void* ptr[4];
            for (uint32_t b = 0; b < 4; ++b)
                if (int rc = resolve(p, l.bindings[b], i, &ptr[b])) return rc;
            cb_attention& a = op.att;
            a.query = static_cast<const float*>(ptr[0]);
            a.key_cache = static_cast<const uint16_t*>(ptr[1]);
            a.value_cache = static_cast<const uint16_t*>(ptr[2]);
            a.out = static_cast<float*>(ptr[3]);
            a.head_dim = static_cast<uint32_t>(override_or(l, "head_dimension", 0.0));
            a.query_heads = static_cast<uint32_t>(override_or(l, "query_heads", 0.0));
            a.kv_heads = static_cast<uint32_t>(override_or(l, "key_value_heads", 0.0));
            a.slots = constant_at<uint32_t>(l, 0);
            a.window = constant_at<uint32_t>(l, 4);
            a.scale_log2e = constant_at<float>(l, 8);
            op.kind = Kind::Attention;
            op.least = 1;
            op.most = UINT32_MAX;
            ops.push_back(op);
            return CB_OK;
        }
        case CB_KERNEL_GATHER: {
            if (!is(entry, "main"))
                return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: gather entry %s has no CUDA form", i, entry);
            if (l.binding_count < 3) return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: gather bindings", i);
            void* ptr[3];
            for (uint32_t b = 0; b < 3; ++b)
                if (int rc = resolve(p, l.bindings[b], i, &ptr[b])) return rc;
            cb_gather& g = op.gather;
            g.piece = ptr[0];
            g.format = l.format;
            g.first_row = constant_at<uint32_t>(l, 0);
            g.row_count = constant_at<uint32_t>(l, 4);
            g.width = constant_at<uint32_t>(l, 8) * 32u;
            g.blocks = constant_at<uint32_t>(l, 12);
            g.scale = constant_at<float>(l, 16);
            g.hidden = static_cast<float*>(ptr[1]);
            g.sampled = static_cast<const uint32_t*>(ptr[2]);
            g.ids = p->step_device->ids;
            op.kind = Kind::Gather;
            ops.push_back(op);
            return CB_OK;
        }
        case CB_KERNEL_TOPK: {
            if (!is(entry, "first"))
                return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: a top-k %s pass without its first", i, entry);
            if (l.binding_count < 2) return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: top-k bindings", i);
            // The passes after it (merge) until the one writing the
            // candidates: one selection over the first pass's logits.
            uint32_t last = i;
            while (last + 1 < count && launches[last + 1].kernel == CB_KERNEL_TOPK &&
                   is(launches[last + 1].entry_point, "merge"))
                ++last;
            if (launches[last].binding_count < 2)
                return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: top-k bindings", last);
            void* logits = nullptr;
            void* cand = nullptr;
            if (int rc = resolve(p, l.bindings[0], i, &logits)) return rc;
            if (int rc = resolve(p, launches[last].bindings[1], last, &cand)) return rc;
            cb_select& s = op.sel;
            s.logits = static_cast<const float*>(logits);
            s.count = constant_at<uint32_t>(l, 0);
            s.candidates = static_cast<uint32_t*>(cand);
            s.rows = 1;
            s.logits_stride = s.count;
            s.candidates_only = 1;
            if (s.count == 0 || s.count > 262144)
                return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: top-k over %u logits", i, s.count);
            op.kind = Kind::Select;
            op.last_launch = last;
            ops.push_back(op);
            i = last;
            return CB_OK;
        }
        case CB_KERNEL_DRAW: {
            if (!is(entry, "main")) return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: draw entry %s", i, entry);
            if (l.binding_count < 2) return fail(CB_ERROR_BUILD, "cb_program_build: launch %u: draw bindings", i);
            void* cand = nullptr;
            void* sampled = nullptr;
            if (int rc = resolve(p, l.bindings[0], i, &cand)) return rc;
            if (int rc = resolve(p, l.bindings[1], i, &sampled)) return rc;
            // Directly after the selection that wrote these candidates, the
            // selection's last CTA draws (one launch for both).
            if (!ops.empty() && ops.back().kind == Kind::Select && !ops.back().select_draws &&
                ops.back().sel.candidates == cand && ops.back().last_token == op.last_token) {
                Op& s = ops.back();
                s.sel.sampled = static_cast<uint32_t*>(sampled);
                s.sel.candidates_only = 0;
                s.select_draws = true;
                s.last_launch = i;
                return CB_OK;
            }
            cb_select_merge& m = op.draw;
            m.lists_data = static_cast<const uint32_t*>(cand);
            m.lists = 1;
            m.rows = 1;
            void* scratch = nullptr;
            if (int rc = dev_alloc(p, &scratch, 128 * sizeof(uint32_t))) return rc;
            m.candidates = static_cast<uint32_t*>(scratch);
            m.sampled = static_cast<uint32_t*>(sampled);
            op.kind = Kind::Draw;
            ops.push_back(op);
            return CB_OK;
        }
        default:
            return fail(CB_ERROR_BUILD, "cb_program_build: launch %u names a kernel (%u, entry %s) with no CUDA form",
                        i, l.kernel, entry);
    }
}

bool runs(const Op& op, const cb_step& s, uint32_t limit) {
    if (op.last_launch >= limit) return false;
    if (s.tokens < op.least || s.tokens > op.most) return false;
    if (op.last_token && !s.logits) return false;
    return true;
}

// One operation with the step's values (tokens, fed, sampling); position,
// identifiers and the fed token come from the device Step.
int launch_op(cb_program* p, const Op& op, const cb_step& s) {
    const uint32_t T = s.tokens;
    const uint32_t* position = &p->step_device->position;
    void* stream = p->stream;
    switch (op.kind) {
        case Kind::Matmul: {
            cb_matmul m = op.mm;
            const float* x = op.x;
            uint32_t tokens = T;
            if (op.decode_form) {
                // matmul.wgsl token_of_decode: the step's last row for a
                // last-token launch (the head), else row 0
                const uint32_t row = op.last_token ? T - 1u : 0u;
                x += static_cast<size_t>(row) * op.x_stride;
                m.gate_input_token = row;
                tokens = 1;
            }
            return cb_matmul_run(&m, x, op.x_stride, tokens, op.out, op.out_stride, CB_MATMUL_PDL, stream);
        }
        case Kind::Norm: {
            cb_norm n = op.norm;
            n.tokens = T;
            return cb_norm_run(&n, CB_RUN_PDL, stream);
        }
        case Kind::Rope: {
            cb_rope r = op.rope;
            r.tokens = T;
            r.position = position;
            return cb_rope_run(&r, CB_RUN_PDL, stream);
        }
        case Kind::Attention: {
            cb_attention a = op.att;
            a.tokens = T;
            a.position = position;
            a.partials = p->partials;
            a.stats = p->stats;
            a.tickets = p->tickets;
            a.max_chunks = p->max_chunks;
            return cb_attention_run(&a, CB_RUN_PDL, stream);
        }
        case Kind::BlockAttention: {
            cb_block_attention a = op.block;
            a.tokens = T;
            return cb_block_attention_run(&a, CB_RUN_PDL, stream);
        }
        case Kind::Pool: {
            cb_pool q = op.pool;
            q.tokens = T;
            return cb_pool_run(&q, CB_RUN_PDL, stream);
        }
        case Kind::Gather: {
            cb_gather g = op.gather;
            g.tokens = T;
            g.fed = s.fed ? 1u : 0u;
            return cb_gather_run(&g, CB_RUN_PDL, stream);
        }
        case Kind::Select: {
            cb_select q = op.sel;
            q.partials = p->sel_partials;
            q.ticket = p->sel_ticket;
            q.position = position;
            q.tokens = T;
            q.seed0 = s.seed[0];
            q.seed1 = s.seed[1];
            q.top_k = s.top_k ? s.top_k : 1u;
            q.temperature = s.temperature;
            q.top_p = s.top_p;
            q.min_p = s.min_p;
            q.log_min_p = s.log_min_p;
            return cb_select_run(&q, CB_RUN_PDL, stream);
        }
        case Kind::Draw: {
            cb_select_merge m = op.draw;
            m.position = position;
            m.tokens = T;
            m.seed0 = s.seed[0];
            m.seed1 = s.seed[1];
            m.top_k = s.top_k ? s.top_k : 1u;
            m.temperature = s.temperature;
            m.top_p = s.top_p;
            m.min_p = s.min_p;
            m.log_min_p = s.log_min_p;
            return cb_select_merge_run(&m, CB_RUN_PDL, stream);
        }
    }
    return fail(CB_ERROR_STEP, "cb_program_run: an operation of no kind");
}

int enqueue_ops(cb_program* p, const cb_step& s, uint32_t limit, Slot* timed, std::vector<uint32_t>* timed_launches) {
    uint32_t mark = 0;
    for (const Op& op : p->ops) {
        if (!runs(op, s, limit)) continue;
        if (int rc = launch_op(p, op, s)) return rc;
        if (timed) {
            if (mark >= timed->marks.size()) {
                cudaEvent_t ev = nullptr;
                const cudaError_t e = cudaEventCreate(&ev);
                if (e != cudaSuccess) return fail_cuda(e, "cb_program_run_profiled: event");
                timed->marks.push_back(ev);
            }
            const cudaError_t e = cudaEventRecord(timed->marks[mark++], p->stream);
            if (e != cudaSuccess) return fail_cuda(e, "cb_program_run_profiled: event");
            timed_launches->push_back(op.last_launch);
        }
    }
    return CB_OK;
}

bool same_graph(const Graph& g, const cb_step& s) {
    return g.logits == (s.logits ? 1u : 0u) && g.fed == (s.fed ? 1u : 0u) && g.seed[0] == s.seed[0] &&
           g.seed[1] == s.seed[1] && g.top_k == s.top_k && g.temperature == s.temperature && g.top_p == s.top_p &&
           g.min_p == s.min_p && g.log_min_p == s.log_min_p;
}

// A one-token step's operations as a graph, captured once for its logits,
// fed and sampling values (the rest comes from the device Step).
int one_token_graph(cb_program* p, const cb_step& s, cudaGraphExec_t* out) {
    for (const Graph& g : p->graphs)
        if (same_graph(g, s)) {
            *out = g.exec;
            return CB_OK;
        }
    if (p->graphs.size() >= 8) {
        cudaGraphExecDestroy(p->graphs.front().exec);
        p->graphs.erase(p->graphs.begin());
    }
    cudaGraph_t graph = nullptr;
    cudaError_t e = cudaStreamBeginCapture(p->stream, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) return fail_cuda(e, "cb_program_run: capture");
    const int rc = enqueue_ops(p, s, UINT32_MAX, nullptr, nullptr);
    const cudaError_t end = cudaStreamEndCapture(p->stream, &graph);
    if (rc != CB_OK) {
        if (graph) cudaGraphDestroy(graph);
        return rc;
    }
    if (end != cudaSuccess) return fail_cuda(end, "cb_program_run: end capture");
    Graph g{};
    g.logits = s.logits ? 1u : 0u;
    g.fed = s.fed ? 1u : 0u;
    g.seed[0] = s.seed[0];
    g.seed[1] = s.seed[1];
    g.top_k = s.top_k;
    g.temperature = s.temperature;
    g.top_p = s.top_p;
    g.min_p = s.min_p;
    g.log_min_p = s.log_min_p;
    e = cudaGraphInstantiate(&g.exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return fail_cuda(e, "cb_program_run: instantiate");
    p->graphs.push_back(g);
    *out = g.exec;
    return CB_OK;
}

// Clears the program's ticket words and the device's fault word after a
// step whose bounded wait ran out (a CTA that gave up may hold a ticket).
void reset_after_fault(cb_program* p) {
    cudaMemsetAsync(p->tickets, 0, p->ticket_words * sizeof(unsigned int), p->stream);
    cudaMemsetAsync(p->sel_ticket, 0, p->sel_ticket_words * sizeof(unsigned int), p->stream);
    if (unsigned int* w = fault_word()) cudaMemsetAsync(w, 0, sizeof(unsigned int), p->stream);
    cudaStreamSynchronize(p->stream);
}

int begin(cb_program* p, const cb_step* step, uint32_t limit, bool profiled, cb_step_callback done,
          cb_profile_callback profile_done, void* userdata) {
    auto refuse = [&](int status, const char* why) {
        if (done) done(status, why, nullptr, 0, userdata);
        if (profile_done) profile_done(status, why, nullptr, 0, 0, 0, nullptr, nullptr, 0, userdata);
        return status;
    };
    if (!step) return refuse(CB_ERROR_INVALID, "a null step");
    if (p->pending.size() >= kOutstanding) return refuse(CB_ERROR_STEP, "a third step while two are outstanding");
    if (profiled && !p->pending.empty() && !p->pending.back().profiled)
        return refuse(CB_ERROR_STEP, "a profiled step beside an unprofiled one");
    if (!profiled && !p->pending.empty() && p->pending.back().profiled)
        return refuse(CB_ERROR_STEP, "a step beside a profiled one");
    if (step->tokens == 0 || step->tokens > kPrefillBlock)
        return refuse(CB_ERROR_INVALID, "a step of 0 or more than 512 tokens");
    Pending o{};
    o.number = p->next_number++;
    o.slot = static_cast<uint32_t>(o.number % kOutstanding);
    o.done = done;
    o.profile_done = profile_done;
    o.userdata = userdata;
    o.profiled = profiled;
    o.reads_back = p->readback && step->logits && limit >= p->launch_count;
    Slot& slot = p->slots[o.slot];
    const uint64_t end_position = static_cast<uint64_t>(step->position) + step->tokens;
    if (end_position > kMaxPositions) {
        o.status = CB_ERROR_STEP;
        o.message = "a step past position 2^24";
    } else if (end_position > static_cast<uint64_t>(p->max_chunks) * 64u) {
        o.status = CB_ERROR_STEP;
        o.message = "a step past the positions the program's attention partials hold";
    }
    *slot.fault_host = 0;
    if (o.status == CB_OK) {
        // The step head, and its identifiers unless it is fed (interface.h Step).
        const bool ids = !step->fed;
        const size_t bytes = kStepHead + (ids ? 4u * ((step->tokens + 3u) / 4u * 4u) : 0u);
        std::memcpy(slot.step_host, step, bytes);
        cudaError_t e = cudaMemcpyAsync(p->step_device, slot.step_host, bytes, cudaMemcpyHostToDevice, p->stream);
        int rc = e == cudaSuccess ? CB_OK : fail_cuda(e, "cb_program_run: the step's parameters");
        if (rc == CB_OK && profiled) {
            if (!slot.begin && (e = cudaEventCreate(&slot.begin)) != cudaSuccess) rc = fail_cuda(e, "event");
            if (rc == CB_OK && (e = cudaEventRecord(slot.begin, p->stream)) != cudaSuccess) rc = fail_cuda(e, "event");
        }
        if (rc == CB_OK) {
            if (profiled) {
                rc = enqueue_ops(p, *step, limit, &slot, &o.timed);
            } else if (step->tokens == 1) {
                cudaGraphExec_t g = nullptr;
                rc = one_token_graph(p, *step, &g);
                if (rc == CB_OK && (e = cudaGraphLaunch(g, p->stream)) != cudaSuccess)
                    rc = fail_cuda(e, "cb_program_run: graph launch");
            } else {
                rc = enqueue_ops(p, *step, limit, nullptr, nullptr);
            }
        }
        if (rc == CB_OK && o.reads_back) {
            e = cudaMemcpyAsync(slot.readback_host, p->readback, p->readback_bytes, cudaMemcpyDeviceToHost, p->stream);
            if (e != cudaSuccess) rc = fail_cuda(e, "cb_program_run: readback");
        }
        if (rc == CB_OK) {
            if (unsigned int* w = fault_word()) {
                e = cudaMemcpyAsync(slot.fault_host, w, sizeof(unsigned int), cudaMemcpyDeviceToHost, p->stream);
                if (e != cudaSuccess) rc = fail_cuda(e, "cb_program_run: fault word");
            }
        }
        if (rc != CB_OK) {
            char msg[1024];
            cb_last_error(msg, sizeof msg);
            o.status = rc;
            o.message = msg;
        }
    }
    const cudaError_t e = cudaEventRecord(slot.done, p->stream);
    if (e != cudaSuccess && o.status == CB_OK) {
        o.status = fail_cuda(e, "cb_program_run: event");
        o.message = "cb_program_run: recording the step's event failed";
    }
    p->pending.push_back(std::move(o));
    return CB_OK;
}

// Settles the oldest step: its event waited on, its fault word read, its
// callback fired.
void settle(cb_program* p) {
    Pending o = std::move(p->pending.front());
    p->pending.pop_front();
    Slot& slot = p->slots[o.slot];
    cudaError_t e = cudaEventSynchronize(slot.done);
    if (e != cudaSuccess && o.status == CB_OK) {
        o.status = fail_cuda(e, "cb_program step");
        char msg[1024];
        cb_last_error(msg, sizeof msg);
        o.message = msg;
    }
    if (o.status == CB_OK && *slot.fault_host) {
        char msg[128];
        std::snprintf(msg, sizeof msg, "a kernel's bounded wait ran out (fault word 0x%x)", *slot.fault_host);
        o.status = CB_ERROR_STEP;
        o.message = msg;
        reset_after_fault(p);
    }
    const bool ok = o.status == CB_OK;
    const void* rb = ok && o.reads_back ? slot.readback_host : nullptr;
    const uint64_t rb_bytes = rb ? p->readback_bytes : 0;
    if (o.profiled) {
        std::vector<uint64_t> ends(o.timed.size(), 0);
        uint64_t end_ns = 0;
        if (ok) {
            for (size_t k = 0; k < o.timed.size(); ++k) {
                float ms = 0.0f;
                cudaEventElapsedTime(&ms, slot.begin, slot.marks[k]);
                ends[k] = static_cast<uint64_t>(static_cast<double>(ms) * 1e6);
            }
            float ms = 0.0f;
            cudaEventElapsedTime(&ms, slot.begin, slot.done);
            end_ns = static_cast<uint64_t>(static_cast<double>(ms) * 1e6);
        }
        if (o.profile_done)
            o.profile_done(o.status, o.message.c_str(), rb, rb_bytes, 0, end_ns, ok ? o.timed.data() : nullptr,
                           ok ? ends.data() : nullptr, ok ? static_cast<uint32_t>(o.timed.size()) : 0u, o.userdata);
    } else if (o.done) {
        o.done(o.status, o.message.c_str(), rb, rb_bytes, o.userdata);
    }
}

}  // namespace

extern "C" {

int cb_buffers_create(const uint64_t* sizes, uint32_t count, cb_buffers** out) {
    if (!out || (count && !sizes)) return fail(CB_ERROR_INVALID, "cb_buffers_create: null argument");
    *out = nullptr;
    cb_buffers* b = new (std::nothrow) cb_buffers();
    if (!b) return fail(CB_ERROR_BUILD, "cb_buffers_create: out of host memory");
    for (uint32_t i = 0; i < count; ++i) {
        void* q = nullptr;
        cudaError_t e = cudaMalloc(&q, sizes[i] ? sizes[i] : 16);
        if (e == cudaSuccess) e = cudaMemset(q, 0, sizes[i] ? sizes[i] : 16);
        if (e != cudaSuccess) {
            if (q) cudaFree(q);
            cb_buffers_destroy(b);
            return fail_cuda(e, "cb_buffers_create");
        }
        b->ptr.push_back(q);
        b->size.push_back(sizes[i]);
    }
    *out = b;
    return CB_OK;
}

void cb_buffers_destroy(cb_buffers* b) {
    if (!b) return;
    for (void* q : b->ptr) cudaFree(q);
    delete b;
}

int cb_buffers_write(cb_buffers* b, uint32_t buffer, uint64_t offset, const void* host, uint64_t bytes) {
    if (!b || !host || buffer >= b->ptr.size()) return fail(CB_ERROR_INVALID, "cb_buffers_write: argument");
    if (offset > b->size[buffer] || bytes > b->size[buffer] - offset)
        return fail(CB_ERROR_INVALID, "cb_buffers_write: %llu bytes at %llu past buffer %u", (unsigned long long)bytes,
                    (unsigned long long)offset, buffer);
    const cudaError_t e =
        cudaMemcpy(static_cast<uint8_t*>(b->ptr[buffer]) + offset, host, bytes, cudaMemcpyHostToDevice);
    return e == cudaSuccess ? CB_OK : fail_cuda(e, "cb_buffers_write");
}

int cb_buffers_read(cb_buffers* b, uint32_t buffer, uint64_t offset, void* host, uint64_t bytes) {
    if (!b || !host || buffer >= b->ptr.size()) return fail(CB_ERROR_INVALID, "cb_buffers_read: argument");
    if (offset > b->size[buffer] || bytes > b->size[buffer] - offset)
        return fail(CB_ERROR_INVALID, "cb_buffers_read: past buffer %u", buffer);
    const cudaError_t e =
        cudaMemcpy(host, static_cast<const uint8_t*>(b->ptr[buffer]) + offset, bytes, cudaMemcpyDeviceToHost);
    return e == cudaSuccess ? CB_OK : fail_cuda(e, "cb_buffers_read");
}

void* cb_buffers_device(const cb_buffers* b, uint32_t buffer) {
    return b && buffer < b->ptr.size() ? b->ptr[buffer] : nullptr;
}

int cb_program_build(cb_buffers* buffers, const cb_launch* launches, uint32_t count, const cb_binding* readback,
                     cb_program** out) {
    if (!buffers || !out || (count && !launches)) return fail(CB_ERROR_INVALID, "cb_program_build: null argument");
    *out = nullptr;
    cb_program* p = new (std::nothrow) cb_program();
    if (!p) return fail(CB_ERROR_BUILD, "cb_program_build: out of host memory");
    p->buffers = buffers;
    p->launch_count = count;
    auto bail = [&](int rc) {
        cb_program_destroy(p);
        return rc;
    };
    cudaError_t e = cudaStreamCreateWithFlags(&p->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) return bail(fail_cuda(e, "cb_program_build: stream"));
    void* step = nullptr;
    if (int rc = dev_alloc(p, &step, sizeof(cb_step))) return bail(rc);
    p->step_device = static_cast<cb_step*>(step);
    if ((e = cudaMemset(step, 0, sizeof(cb_step))) != cudaSuccess) return bail(fail_cuda(e, "cb_program_build"));
    for (uint32_t i = 0; i < count; ++i)
        if (int rc = build_one(p, launches, count, i, p->ops)) return bail(rc);
    // The program's own scratch: attention partials for every 64-key chunk
    // the largest cache reaches, for a whole step's rows; the selection's
    // per-tile candidates; the ticket words (left zero after each run).
    uint32_t max_slots = 0, max_q = 0, max_d = 0, max_kv = 0, max_count = 0;
    for (const Op& op : p->ops) {
        if (op.kind == Kind::Attention) {
            max_slots = std::max(max_slots, op.att.slots);
            max_q = std::max(max_q, op.att.query_heads);
            max_kv = std::max(max_kv, op.att.kv_heads);
            max_d = std::max(max_d, op.att.head_dim);
        }
        if (op.kind == Kind::Select) max_count = std::max(max_count, op.sel.count);
    }
    p->max_chunks = max_slots ? (max_slots + 63u) / 64u : kMaxPositions / 64u;
    if (max_q) {
        const size_t rows = static_cast<size_t>(p->max_chunks) * kPrefillBlock * max_q;
        void* q = nullptr;
        if (int rc = dev_alloc(p, &q, rows * max_d * sizeof(float))) return bail(rc);
        p->partials = static_cast<float*>(q);
        if (int rc = dev_alloc(p, &q, rows * 2 * sizeof(float))) return bail(rc);
        p->stats = static_cast<float*>(q);
        p->ticket_words = std::max(cb_attention_tickets(kPrefillBlock, max_q, max_kv), max_kv);
        if (int rc = dev_alloc(p, &q, p->ticket_words * sizeof(unsigned int))) return bail(rc);
        p->tickets = static_cast<unsigned int*>(q);
        if ((e = cudaMemset(q, 0, p->ticket_words * sizeof(unsigned int))) != cudaSuccess)
            return bail(fail_cuda(e, "cb_program_build"));
    }
    if (max_count) {
        void* q = nullptr;
        if (int rc = dev_alloc(p, &q, static_cast<size_t>(cb_select_tiles(max_count)) * 128 * sizeof(uint32_t)))
            return bail(rc);
        p->sel_partials = static_cast<uint32_t*>(q);
        p->sel_ticket_words = cb_select_tickets(max_count);
        if (int rc = dev_alloc(p, &q, p->sel_ticket_words * sizeof(unsigned int))) return bail(rc);
        p->sel_ticket = static_cast<unsigned int*>(q);
        if ((e = cudaMemset(q, 0, p->sel_ticket_words * sizeof(unsigned int))) != cudaSuccess)
            return bail(fail_cuda(e, "cb_program_build"));
    }
    if (readback) {
        if (readback->size > kMaxReadback || readback->size % 4 != 0)
            return bail(fail(CB_ERROR_BUILD, "cb_program_build: a readback of %llu bytes (at most 4096, whole words)",
                             static_cast<unsigned long long>(readback->size)));
        void* rb = nullptr;
        if (int rc = resolve(p, *readback, count, &rb)) return bail(rc);
        p->readback = rb;
        p->readback_bytes = readback->size;
    }
    for (Slot& s : p->slots) {
        if ((e = cudaMallocHost(reinterpret_cast<void**>(&s.step_host), sizeof(cb_step))) != cudaSuccess ||
            (e = cudaMallocHost(reinterpret_cast<void**>(&s.readback_host), kMaxReadback)) != cudaSuccess ||
            (e = cudaMallocHost(reinterpret_cast<void**>(&s.fault_host), sizeof(unsigned int))) != cudaSuccess ||
            (e = cudaEventCreateWithFlags(&s.done, cudaEventDefault)) != cudaSuccess)
            return bail(fail_cuda(e, "cb_program_build: host slots"));
    }
    *out = p;
    return CB_OK;
}

int cb_program_run(cb_program* p, const cb_step* step, cb_step_callback done, void* userdata) {
    if (!p) return fail(CB_ERROR_INVALID, "cb_program_run: null program");
    return begin(p, step, UINT32_MAX, false, done, nullptr, userdata);
}

int cb_program_run_profiled(cb_program* p, const cb_step* step, uint32_t launches, cb_profile_callback done,
                            void* userdata) {
    if (!p) return fail(CB_ERROR_INVALID, "cb_program_run_profiled: null program");
    if (launches > p->launch_count) {
        if (done) done(CB_ERROR_STEP, "more launches than the graph has", nullptr, 0, 0, 0, nullptr, nullptr, 0, userdata);
        return CB_ERROR_STEP;
    }
    return begin(p, step, launches, true, nullptr, done, userdata);
}

int cb_program_poll(cb_program* p, uint32_t wait) {
    if (!p) return fail(CB_ERROR_INVALID, "cb_program_poll: null program");
    int fired = 0;
    while (!p->pending.empty()) {
        if (!(wait && fired == 0)) {
            const cudaError_t q = cudaEventQuery(p->slots[p->pending.front().slot].done);
            if (q == cudaErrorNotReady) break;
        }
        settle(p);
        ++fired;
    }
    return fired;
}

uint32_t cb_program_outstanding(const cb_program* p) { return p ? static_cast<uint32_t>(p->pending.size()) : 0u; }

uint32_t cb_program_launch_count(const cb_program* p) { return p ? p->launch_count : 0u; }

void* cb_program_stream(const cb_program* p) { return p ? static_cast<void*>(p->stream) : nullptr; }

void cb_program_destroy(cb_program* p) {
    if (!p) return;
    if (p->stream) cudaStreamSynchronize(p->stream);
    while (!p->pending.empty()) {
        Pending o = std::move(p->pending.front());
        p->pending.pop_front();
        const char* why = "the program was destroyed with the step in flight";
        if (o.profiled && o.profile_done)
            o.profile_done(CB_ERROR_CANCELLED, why, nullptr, 0, 0, 0, nullptr, nullptr, 0, o.userdata);
        else if (o.done)
            o.done(CB_ERROR_CANCELLED, why, nullptr, 0, o.userdata);
    }
    for (Graph& g : p->graphs)
        if (g.exec) cudaGraphExecDestroy(g.exec);
    for (Slot& s : p->slots) {
        if (s.step_host) cudaFreeHost(s.step_host);
        if (s.readback_host) cudaFreeHost(s.readback_host);
        if (s.fault_host) cudaFreeHost(s.fault_host);
        if (s.done) cudaEventDestroy(s.done);
        if (s.begin) cudaEventDestroy(s.begin);
        for (cudaEvent_t ev : s.marks) cudaEventDestroy(ev);
    }
    for (void* q : p->owned) cudaFree(q);
    if (p->stream) cudaStreamDestroy(p->stream);
    delete p;
}

}  // extern "C"
