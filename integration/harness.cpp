// A model file loaded the way the reference's runtime loads one, run on the
// CUDA backend — for the integration tests (tests/test_program_gpu.py) and
// as a worked example of the drop-in: the file's index read by the
// reference's GGUF reader, its architecture's description, the residency
// plan, the routes and piece writer of the upload, the architecture's
// decoder graph of kernels::Launch — all the reference's own code — then
// residency::cuda::Upload and kernels::cuda::Program (program_cuda.h) in
// place of the WebGPU ones.
//
// A plain C interface, for ctypes: cbh_open, cbh_run (enqueue a step),
// cbh_poll (the finished steps' records, in run order), cbh_logits,
// cbh_profile, cbh_close.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <memory>
#include <string>
#include <vector>

#include "charlotte_b200.h"
#include "core/arch/architecture.h"
#include "core/capability/capability.h"
#include "core/gguf/byte_source.h"
#include "core/gguf/reader.h"
#include "core/graph/encoder.h"
#include "core/graph/graph.h"
#include "core/policy/policy.h"
#include "program_cuda.h"

using namespace bllm;

namespace {

// WebGPU's default limits (the reference's own tests plan with these), so
// the plan — its buffers, and which weights split into pieces — is the one
// the reference makes.
constexpr residency::DeviceLimits kLimits{256ull << 20, 128ull << 20, 256};

struct Result {
    std::uint32_t tag;
    std::int32_t status;
    std::uint32_t record[4];
};

}  // namespace

struct cbh {
    std::vector<std::byte> file;
    gguf::TensorIndex index;
    model::ModelDescription model{};
    residency::ResidencyPlan plan;
    std::unique_ptr<residency::cuda::Upload> upload;
    std::unique_ptr<kernels::cuda::Program> program;
    residency::BufferRange logits{}, sampled{}, embedding{};
    bool encoder = false;
    std::uint32_t launches = 0;
    std::vector<Result> results;
    std::string message;
    // run_profiled's answer
    std::uint64_t profile_end_ns = 0;
    std::vector<std::pair<std::uint32_t, std::uint64_t>> profile_launches;
};

namespace {

int fail(cbh* h, char* err, std::size_t len, const std::string& why) {
    if (err && len) std::snprintf(err, len, "%s", why.c_str());
    delete h;
    return CB_ERROR_BUILD;
}

struct Built {
    std::unique_ptr<kernels::cuda::Program> program;
    std::string message;
};

void on_built(std::unique_ptr<kernels::cuda::Program> p, kernels::cuda::ProgramError e, std::string_view message,
              void* userdata) {
    auto* b = static_cast<Built*>(userdata);
    if (e == kernels::cuda::ProgramError::Ok) b->program = std::move(p);
    b->message = std::string(message);
}

void on_step(kernels::cuda::ProgramError e, std::string_view message, std::span<const std::byte> readback,
             void* userdata) {
    auto* pair = static_cast<std::pair<cbh*, std::uint32_t>*>(userdata);
    cbh* h = pair->first;
    Result r{pair->second, static_cast<std::int32_t>(e), {0, 0, 0, 0}};
    if (readback.size() >= 16) std::memcpy(r.record, readback.data(), 16);
    if (e != kernels::cuda::ProgramError::Ok) h->message = std::string(message);
    h->results.push_back(r);
    delete pair;
}

void on_profiled(kernels::cuda::ProgramError e, std::string_view message, std::span<const std::byte> readback,
                 const kernels::cuda::Program::Timestamps& times, void* userdata) {
    auto* pair = static_cast<std::pair<cbh*, std::uint32_t>*>(userdata);
    cbh* h = pair->first;
    Result r{pair->second, static_cast<std::int32_t>(e), {0, 0, 0, 0}};
    if (readback.size() >= 16) std::memcpy(r.record, readback.data(), 16);
    if (e != kernels::cuda::ProgramError::Ok) h->message = std::string(message);
    h->results.push_back(r);
    h->profile_end_ns = times.end_ns;
    h->profile_launches.assign(times.launches.begin(), times.launches.end());
    delete pair;
}

kernels::Step step_of(const std::uint32_t* ids, std::uint32_t tokens, std::uint32_t position, std::uint32_t logits,
                      std::uint32_t fed, const float* sampling, std::uint32_t top_k, std::uint32_t seed0,
                      std::uint32_t seed1) {
    kernels::Step s{};
    s.position = position;
    s.tokens = tokens;
    s.logits = logits;
    s.fed = fed;
    s.seed[0] = seed0;
    s.seed[1] = seed1;
    s.top_k = top_k;
    s.temperature = sampling ? sampling[0] : 0.0f;
    s.top_p = sampling ? sampling[1] : 1.0f;
    s.min_p = sampling ? sampling[2] : 0.0f;
    s.log_min_p = s.min_p > 0.0f ? std::log(s.min_p) : 0.0f;
    if (!fed && ids)
        for (std::uint32_t i = 0; i < tokens && i < s.ids.size(); ++i) s.ids[i] = ids[i];
    return s;
}

}  // namespace

extern "C" {

__attribute__((visibility("default"))) int cbh_open(const char* path, std::uint32_t max_chunk, cbh** out, char* err,
                                                    std::size_t err_len) {
    *out = nullptr;
    auto* h = new cbh();
    std::ifstream f(path, std::ios::binary | std::ios::ate);
    if (!f) return fail(h, err, err_len, std::string("cannot open ") + path);
    h->file.resize(static_cast<std::size_t>(f.tellg()));
    f.seekg(0);
    f.read(reinterpret_cast<char*>(h->file.data()), static_cast<std::streamsize>(h->file.size()));
    gguf::MemoryByteSource source{std::span<const std::byte>(h->file)};
    if (const gguf::ReadResult r = gguf::read_index(source, h->index); r.error != gguf::ReadError::Ok)
        return fail(h, err, err_len, "read_index failed");
    std::string_view name;
    if (h->index.read_string("general.architecture", name) != gguf::MetadataError::Ok)
        return fail(h, err, err_len, "no general.architecture");
    const arch::Architecture* a = capability::find_architecture(name);
    if (!a || (!arch::decoder_graph(*a) && !arch::encoder_graph(*a)))
        return fail(h, err, err_len, "no architecture " + std::string(name));
    h->encoder = arch::encoder_graph(*a) != nullptr;
    if (const auto r = a->describe(h->index, h->model); !r.ok()) return fail(h, err, err_len, "describe: " + r.subject);
    if (const auto r = residency::plan_residency(h->index, h->model, kLimits, policy::LoadPolicy{},
                                                 h->encoder ? graph::encoder_working_set(h->model)
                                                            : graph::decoder_working_set(h->model),
                                                 h->plan);
        !r.ok())
        return fail(h, err, err_len, "plan: " + r.subject);
    if (const auto r = residency::cuda::Upload::begin(h->index, h->plan, h->file.size(), capability::find_format, {},
                                                      max_chunk, h->upload);
        !r.ok())
        return fail(h, err, err_len, "upload: " + r.subject);
    // the file in chunks of max_chunk, in order, as a loader reads it
    for (std::uint64_t at = 0; at < h->file.size(); at += max_chunk) {
        const std::size_t n = static_cast<std::size_t>(std::min<std::uint64_t>(max_chunk, h->file.size() - at));
        if (const auto r = h->upload->accept(at, std::span<const std::byte>(h->file.data() + at, n)); !r.ok())
            return fail(h, err, err_len, "upload accept: " + r.subject);
    }
    if (const auto r = h->upload->finish(h->file.size()); !r.ok())
        return fail(h, err, err_len, "upload finish: " + r.subject);
    const residency::ResidencyPlan& plan = h->upload->plan();
    std::vector<kernels::Launch> launches;
    const formats::Format* f16 = capability::find_format(gguf::TensorType::F16);
    // An encoder's one step ends in the pooled, unit-length vector, which it
    // reads back (runtime/embedder.h); a decoder's in the sampled record.
    if (const auto r = h->encoder ? arch::encoder_graph(*a)(h->model, plan, launches)
                                  : arch::decoder_graph(*a)(h->model, plan, *f16, launches);
        !r.ok())
        return fail(h, err, err_len, "graph: " + r.subject);
    for (const residency::PlannedScratch& s : plan.scratch) {
        if (s.purpose == "logits") h->logits = s.range;
        if (s.purpose == "sampled") h->sampled = s.range;
        if (s.purpose == "embedding") h->embedding = s.range;
    }
    h->launches = static_cast<std::uint32_t>(launches.size());
    const residency::BufferRange& back = h->encoder ? h->embedding : h->sampled;
    Built built;
    kernels::cuda::Program::build(*h->upload, std::move(launches),
                                  kernels::Binding{back.buffer, back.offset, back.length}, on_built, &built);
    if (!built.program) return fail(h, err, err_len, "build: " + built.message);
    h->program = std::move(built.program);
    *out = h;
    return CB_OK;
}

__attribute__((visibility("default"))) std::uint32_t cbh_vocab(const cbh* h) { return h->model.vocabulary_size; }
// An encoder's embedding length (0 for a decoder).
__attribute__((visibility("default"))) std::uint32_t cbh_embedding_length(const cbh* h) {
    return h->encoder ? h->model.encoder->embedding_length : 0u;
}
__attribute__((visibility("default"))) std::uint32_t cbh_launches(const cbh* h) { return h->launches; }
__attribute__((visibility("default"))) std::uint32_t cbh_context(const cbh* h) { return h->plan.context_offered; }

// Enqueues a step (Program::run); its record arrives through cbh_poll with
// `tag`. sampling: temperature, top_p, min_p (NULL: greedy).
__attribute__((visibility("default"))) int cbh_run(cbh* h, const std::uint32_t* ids, std::uint32_t tokens,
                                                   std::uint32_t position, std::uint32_t logits, std::uint32_t fed,
                                                   const float* sampling, std::uint32_t top_k, std::uint32_t seed0,
                                                   std::uint32_t seed1, std::uint32_t tag) {
    const kernels::Step s = step_of(ids, tokens, position, logits, fed, sampling, top_k, seed0, seed1);
    h->program->run(s, on_step, new std::pair<cbh*, std::uint32_t>(h, tag));
    return CB_OK;
}

// The records of steps finished so far (with `wait`, at least the oldest
// outstanding one's), in the order they were run: rows of {tag, status,
// token, failed, u, 0}.
__attribute__((visibility("default"))) int cbh_poll(cbh* h, std::uint32_t wait, std::uint32_t* out,
                                                    std::uint32_t capacity) {
    h->program->process_events(wait != 0);
    const std::uint32_t n = std::min<std::uint32_t>(capacity, static_cast<std::uint32_t>(h->results.size()));
    for (std::uint32_t i = 0; i < n; ++i) {
        const Result& r = h->results[i];
        out[6 * i + 0] = r.tag;
        out[6 * i + 1] = static_cast<std::uint32_t>(r.status);
        std::memcpy(out + 6 * i + 2, r.record, 16);
    }
    h->results.erase(h->results.begin(), h->results.begin() + n);
    return static_cast<int>(n);
}

__attribute__((visibility("default"))) std::uint32_t cbh_outstanding(const cbh* h) { return h->program->outstanding(); }

__attribute__((visibility("default"))) const char* cbh_message(const cbh* h) { return h->message.c_str(); }

// The last step's logits (the plan's logits buffer) to host memory.
__attribute__((visibility("default"))) int cbh_logits(cbh* h, float* out) {
    return cb_buffers_read(h->upload->buffers(), static_cast<std::uint32_t>(h->logits.buffer), h->logits.offset, out,
                           std::uint64_t{h->model.vocabulary_size} * 4);
}

// An encoder's last step's embedding (the plan's embedding buffer) to host
// memory, embedding-length floats.
__attribute__((visibility("default"))) int cbh_embedding(cbh* h, float* out) {
    if (!h->encoder) return CB_ERROR_INVALID;
    return cb_buffers_read(h->upload->buffers(), static_cast<std::uint32_t>(h->embedding.buffer), h->embedding.offset,
                           out, std::uint64_t{h->model.encoder->embedding_length} * 4);
}

// Any scratch buffer of the plan by its purpose ("hidden", "per_layer", …):
// `count` floats from its start to host memory (for tests that check a step
// part of the way).
__attribute__((visibility("default"))) int cbh_scratch(cbh* h, const char* purpose, float* out, std::uint64_t count) {
    for (const residency::PlannedScratch& s : h->upload->plan().scratch)
        if (s.purpose == purpose)
            return cb_buffers_read(h->upload->buffers(), static_cast<std::uint32_t>(s.range.buffer), s.range.offset,
                                   out, std::min<std::uint64_t>(count * 4, s.range.length));
    return CB_ERROR_INVALID;
}

// A profiled step of its first `launches` launches, waited on: the number
// of timed launches, each launch's index and end (ns from the step's begin)
// into index/end_ns (capacity entries), the step's end into *step_ns.
__attribute__((visibility("default"))) int cbh_profile(cbh* h, const std::uint32_t* ids, std::uint32_t tokens,
                                                       std::uint32_t position, std::uint32_t logits,
                                                       std::uint32_t launches, std::uint32_t* index,
                                                       std::uint64_t* end_ns, std::uint32_t capacity,
                                                       std::uint64_t* step_ns, std::int32_t* status) {
    const kernels::Step s = step_of(ids, tokens, position, logits, 0, nullptr, 1, 0, 0);
    h->program->run_profiled(s, launches, on_profiled, new std::pair<cbh*, std::uint32_t>(h, 0xFFFFFFFFu));
    h->program->process_events(true);
    *status = h->results.empty() ? -1 : h->results.back().status;
    h->results.clear();
    *step_ns = h->profile_end_ns;
    const std::uint32_t n = std::min<std::uint32_t>(capacity, static_cast<std::uint32_t>(h->profile_launches.size()));
    for (std::uint32_t i = 0; i < n; ++i) {
        index[i] = h->profile_launches[i].first;
        end_ns[i] = h->profile_launches[i].second;
    }
    return static_cast<int>(h->profile_launches.size());
}

__attribute__((visibility("default"))) void cbh_close(cbh* h) {
    if (!h) return;
    h->program.reset();   // outstanding steps fire Cancelled into h->results
    h->upload.reset();
    delete h;
}

}  // extern "C"
