// residency::Upload and kernels::Program over CUDA (program_cuda.h): the
// reference's plan, routes, piece writer and launch descriptions, carried
// out by libcharlotte_b200.
#include "program_cuda.h"

#include <cstddef>
#include <cstring>
#include <utility>

#include "bllm/shaders_generated.h"
#include "core/residency/piece_writer.h"

namespace bllm::residency::cuda {

namespace {

UploadError from_route(RouteError e) {
    switch (e) {
        case RouteError::Ok: return UploadError::Ok;
        case RouteError::UnsupportedFormat: return UploadError::UnsupportedFormat;
        case RouteError::OutOfRange: return UploadError::OutOfRange;
        case RouteError::NotACandidate: return UploadError::NotACandidate;
        case RouteError::RowNotSteppable: return UploadError::RowNotSteppable;
    }
    return UploadError::OutOfRange;
}

UploadError from_write(WriteError e) {
    switch (e) {
        case WriteError::Ok: return UploadError::Ok;
        case WriteError::OutOfOrder: return UploadError::OutOfOrder;
        case WriteError::ChunkTooLarge: return UploadError::ChunkTooLarge;
        case WriteError::Unfinished: return UploadError::Unfinished;
    }
    return UploadError::OutOfOrder;
}

std::string last_error() {
    char buf[1024];
    cb_last_error(buf, sizeof buf);
    return buf;
}

}  // namespace

struct Upload::Writer {
    Writer(std::span<const Route> routes, std::size_t max_chunk, std::span<const FileRange> ranges)
        : writer(routes, max_chunk, ranges) {}
    PieceWriter writer;
    std::vector<Write> writes;
};

UploadResult Upload::begin(const gguf::TensorIndex& index, const ResidencyPlan& plan, std::uint64_t file_size,
                           FindFormat find_format, std::span<const gguf::TensorId> confirmed_duplicates,
                           std::size_t max_chunk, std::unique_ptr<Upload>& out, std::span<const FileRange> ranges) {
    std::unique_ptr<Upload> u(new Upload());
    if (const RouteResult r =
            plan_routes(index, plan, file_size, find_format, confirmed_duplicates, u->routes_, u->plan_, ranges);
        !r.ok()) {
        return {from_route(r.error), r.subject};
    }
    std::vector<std::uint64_t> sizes;
    sizes.reserve(u->plan_.buffers.size());
    for (const PlannedBuffer& b : u->plan_.buffers) sizes.push_back(b.size);
    if (cb_buffers_create(sizes.data(), static_cast<std::uint32_t>(sizes.size()), &u->buffers_) != CB_OK)
        return {UploadError::OutOfMemory, last_error()};
    u->writer_ = std::make_unique<Writer>(u->routes_, max_chunk, ranges);
    out = std::move(u);
    return {};
}

UploadResult Upload::accept(std::uint64_t file_offset, std::span<const std::byte> chunk) {
    writer_->writes.clear();
    if (const WriteError e = writer_->writer.accept(file_offset, chunk, writer_->writes); e != WriteError::Ok)
        return {from_write(e), "chunk at " + std::to_string(file_offset)};
    for (const Write& w : writer_->writes) {
        if (cb_buffers_write(buffers_, static_cast<std::uint32_t>(w.buffer), w.offset, w.bytes.data(),
                             w.bytes.size()) != CB_OK)
            return {UploadError::OutOfRange, last_error()};
    }
    return {};
}

UploadResult Upload::finish(std::uint64_t file_size) {
    if (const WriteError e = writer_->writer.finish(file_size); e != WriteError::Ok) return {from_write(e), "finish"};
    return {};
}

void* Upload::buffer(BufferIndex index) const noexcept {
    return cb_buffers_device(buffers_, static_cast<std::uint32_t>(index));
}

Upload::~Upload() { cb_buffers_destroy(buffers_); }

}  // namespace bllm::residency::cuda

namespace bllm::kernels::cuda {

namespace {

static_assert(sizeof(cb_step) == sizeof(Step), "cb_step is interface.h's Step byte for byte");
static_assert(offsetof(cb_step, ids) == offsetof(Step, ids));
static_assert(offsetof(cb_step, log_min_p) == offsetof(Step, log_min_p));

ProgramError from_status(int status) {
    switch (status) {
        case CB_OK: return ProgramError::Ok;
        case CB_ERROR_BUILD: return ProgramError::Build;
        case CB_ERROR_DEVICE_LOST: return ProgramError::DeviceLost;
        case CB_ERROR_CANCELLED: return ProgramError::Cancelled;
        default: return ProgramError::Step;
    }
}

cb_binding binding_of(const Binding& b) {
    return {static_cast<std::uint32_t>(b.buffer), 0u, b.offset, b.size};
}

struct StepContext {
    StepCallback done;
    Program::ProfileCallback profile_done;
    void* userdata;
};

void step_done(int status, const char* message, const void* readback, std::uint64_t bytes, void* userdata) {
    std::unique_ptr<StepContext> c(static_cast<StepContext*>(userdata));
    c->done(from_status(status), message ? std::string_view(message) : std::string_view(),
            std::span<const std::byte>(static_cast<const std::byte*>(readback), readback ? bytes : 0), c->userdata);
}

void profile_done(int status, const char* message, const void* readback, std::uint64_t bytes, std::uint64_t begin_ns,
                  std::uint64_t end_ns, const std::uint32_t* index, const std::uint64_t* ends, std::uint32_t n,
                  void* userdata) {
    std::unique_ptr<StepContext> c(static_cast<StepContext*>(userdata));
    std::vector<std::pair<std::uint32_t, std::uint64_t>> launches(n);
    for (std::uint32_t i = 0; i < n; ++i) launches[i] = {index[i], ends[i]};
    c->profile_done(from_status(status), message ? std::string_view(message) : std::string_view(),
                    std::span<const std::byte>(static_cast<const std::byte*>(readback), readback ? bytes : 0),
                    Program::Timestamps{begin_ns, end_ns, launches}, c->userdata);
}

}  // namespace

std::uint32_t kernel_of(const Launch& l) noexcept {
    if (l.kernel == shaders::matmul) return CB_KERNEL_MATMUL;
    if (l.kernel == shaders::norm) return CB_KERNEL_NORM;
    if (l.kernel == shaders::attention) return CB_KERNEL_ATTENTION;
    if (l.kernel == shaders::gather) return CB_KERNEL_GATHER;
    if (l.kernel == shaders::topk) return CB_KERNEL_TOPK;
    if (l.kernel == shaders::draw) return CB_KERNEL_DRAW;
    // rope.cpp joins the shared rope.wgsl with a form's entry point
    if (l.kernel.size() == shaders::rope.size() + shaders::rope_cache.size() && l.kernel.starts_with(shaders::rope) &&
        l.kernel.ends_with(shaders::rope_cache))
        return CB_KERNEL_ROPE_CACHE;
    if (l.kernel.size() == shaders::rope.size() + shaders::rope_encode.size() && l.kernel.starts_with(shaders::rope) &&
        l.kernel.ends_with(shaders::rope_encode))
        return CB_KERNEL_ROPE_ENCODE;
    if (l.kernel == shaders::block_attention) return CB_KERNEL_BLOCK_ATTENTION;
    if (l.kernel == shaders::pool) return CB_KERNEL_POOL;
    return CB_KERNEL_UNKNOWN;
}

void Program::build(const residency::cuda::Upload& upload, std::vector<Launch> launches,
                    std::optional<Binding> readback, BuildCallback done, void* userdata) {
    // Each launch in plain C: the strings NUL-terminated and every array
    // held here for the call (the library keeps none of it).
    std::vector<std::string> names;
    std::vector<std::vector<cb_binding>> bindings(launches.size());
    std::vector<std::vector<cb_override>> overrides(launches.size());
    std::vector<cb_launch> out(launches.size());
    std::size_t strings = launches.size();
    for (const Launch& l : launches) strings += l.overrides.size();
    names.reserve(strings);
    for (std::size_t i = 0; i < launches.size(); ++i) {
        const Launch& l = launches[i];
        for (const Binding& b : l.bindings) bindings[i].push_back(binding_of(b));
        names.emplace_back(l.entry_point);
        const char* entry = names.back().c_str();
        for (const Override& o : l.overrides) {
            names.emplace_back(o.name);
            overrides[i].push_back({names.back().c_str(), o.value});
        }
        cb_launch& c = out[i];
        c.kernel = kernel_of(l);
        c.entry_point = entry;
        c.format = l.format ? static_cast<std::uint32_t>(l.format->type()) : CB_NO_FORMAT;
        c.pack_format = l.pack_format ? static_cast<std::uint32_t>(l.pack_format->type()) : CB_NO_FORMAT;
        c.constants = reinterpret_cast<const std::uint8_t*>(l.constants.data());
        c.constants_bytes = static_cast<std::uint32_t>(l.constants.size());
        c.bindings = bindings[i].data();
        c.binding_count = static_cast<std::uint32_t>(bindings[i].size());
        c.invocations_per_row = l.invocations_per_row;
        c.workgroup_size = l.workgroup_size;
        c.rows = l.rows == Rows::LastToken ? CB_ROWS_LAST_TOKEN : CB_ROWS_EVERY_TOKEN;
        c.overrides = overrides[i].data();
        c.override_count = static_cast<std::uint32_t>(overrides[i].size());
        c.rows_per_tile = l.rows_per_tile;
        c.key_split = l.key_split == KeySplit::PerChunk    ? CB_KEY_SPLIT_PER_CHUNK
                      : l.key_split == KeySplit::WhenSplit ? CB_KEY_SPLIT_WHEN_SPLIT
                                                           : CB_KEY_SPLIT_NONE;
        c.window = l.window;
        c.partial_rows = l.partial_rows;
        c.tokens_least = l.tokens.least;
        c.tokens_most = l.tokens.most;
        c.row_divisor = l.row_divisor;
    }
    cb_binding rb{};
    if (readback) rb = binding_of(*readback);
    std::unique_ptr<Program> p(new Program());
    const int rc = cb_program_build(upload.buffers(), out.data(), static_cast<std::uint32_t>(out.size()),
                                    readback ? &rb : nullptr, &p->program_);
    if (rc != CB_OK) {
        char msg[1024];
        cb_last_error(msg, sizeof msg);
        done(nullptr, from_status(rc), msg, userdata);
        return;
    }
    done(std::move(p), ProgramError::Ok, {}, userdata);
}

void Program::run(const Step& step, StepCallback done, void* userdata) {
    auto* c = new StepContext{done, nullptr, userdata};
    cb_step s;
    std::memcpy(&s, &step, sizeof s);
    cb_program_run(program_, &s, step_done, c);
}

void Program::run_profiled(const Step& step, std::uint32_t launches, ProfileCallback done, void* userdata) {
    auto* c = new StepContext{nullptr, done, userdata};
    cb_step s;
    std::memcpy(&s, &step, sizeof s);
    cb_program_run_profiled(program_, &s, launches, profile_done, c);
}

std::uint32_t Program::launch_count() const noexcept { return cb_program_launch_count(program_); }

int Program::process_events(bool wait) { return cb_program_poll(program_, wait ? 1u : 0u); }

std::uint32_t Program::outstanding() const noexcept { return cb_program_outstanding(program_); }

Program::~Program() { cb_program_destroy(program_); }

}  // namespace bllm::kernels::cuda
