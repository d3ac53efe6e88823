// The reference's residency::Upload and kernels::Program over CUDA, for a
// CUDA build of plainsight-systems/charlotte. They keep the interfaces of
// src/core/residency/upload.h:245-332 and src/core/kernels/program.h:
// 262-331 — the plan, the routes, the launchers' kernels::Launch lists and
// kernels::Step are the reference's own types, compiled from its sources —
// with the WebGPU device, buffers, pipelines and queue replaced by the C ABI
// of libcharlotte_b200 (include/charlotte_b200.h: cb_buffers, cb_program).
//
// What changes for a caller: Upload is made and fed synchronously (CUDA has
// no mapping to wait for), and a program's callbacks fire from
// process_events(), which stands where the runtime's wgpuInstanceProcessEvents
// stands (the reference's callbacks run inside it too).
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <optional>
#include <span>
#include <string>
#include <string_view>
#include <vector>

#include "charlotte_b200.h"
#include "core/gguf/index.h"
#include "core/kernels/interface.h"
#include "core/residency/file_ranges.h"
#include "core/residency/plan.h"
#include "core/residency/routes.h"

namespace bllm::residency::cuda {

// upload.h UploadError's meanings this path can reach.
enum class UploadError {
    Ok,
    UnsupportedFormat,
    OutOfRange,
    NotACandidate,
    RowNotSteppable,
    OutOfMemory,
    OutOfOrder,
    ChunkTooLarge,
    Unfinished,
};

struct UploadResult {
    UploadError error = UploadError::Ok;
    std::string subject;
    [[nodiscard]] bool ok() const noexcept { return error == UploadError::Ok; }
};

// The plan's buffers on the device, its weights written from the file's
// bytes as they arrive (upload.h: routes planned by plan_routes, each
// piece's streams and Q6_K repack written by PieceWriter), working buffers
// and caches zeroed.
class Upload {
public:
    // upload.h Upload::begin: plans the routes and creates the buffers.
    static UploadResult begin(const gguf::TensorIndex& index, const ResidencyPlan& plan, std::uint64_t file_size,
                              FindFormat find_format, std::span<const gguf::TensorId> confirmed_duplicates,
                              std::size_t max_chunk, std::unique_ptr<Upload>& out,
                              std::span<const FileRange> ranges = {});
    // A chunk of the file, in order from its first byte (upload.h accept).
    UploadResult accept(std::uint64_t file_offset, std::span<const std::byte> chunk);
    // The file's end: every route filled (upload.h finish).
    UploadResult finish(std::uint64_t file_size);

    [[nodiscard]] const ResidencyPlan& plan() const noexcept { return plan_; }
    [[nodiscard]] cb_buffers* buffers() const noexcept { return buffers_; }
    [[nodiscard]] void* buffer(BufferIndex index) const noexcept;

    ~Upload();
    Upload(const Upload&) = delete;
    Upload& operator=(const Upload&) = delete;

private:
    Upload() = default;
    struct Writer;
    ResidencyPlan plan_;
    std::vector<Route> routes_;
    cb_buffers* buffers_ = nullptr;
    std::unique_ptr<Writer> writer_;
};

}  // namespace bllm::residency::cuda

namespace bllm::kernels::cuda {

// program.h ProgramError.
enum class ProgramError { Ok, Build, Step, DeviceLost, Cancelled };

class Program;

using BuildCallback = void (*)(std::unique_ptr<Program> program, ProgramError error, std::string_view message,
                               void* userdata);
using StepCallback = void (*)(ProgramError error, std::string_view message, std::span<const std::byte> readback,
                              void* userdata);

// The kernel a launch names, by the embedded WGSL source it carries.
[[nodiscard]] std::uint32_t kernel_of(const Launch& launch) noexcept;

class Program {
public:
    // program.h Program::build. `done` is called once, before this returns.
    static void build(const residency::cuda::Upload& upload, std::vector<Launch> launches,
                      std::optional<Binding> readback, BuildCallback done, void* userdata);

    // program.h Program::run: enqueued, `done` fired by process_events in
    // run order; a third step while two are outstanding fails at once.
    void run(const Step& step, StepCallback done, void* userdata);

    // program.h Program::run_profiled, launch_count, can_profile: the first
    // `launches` launches of a step, each timed by CUDA events.
    struct Timestamps {
        std::uint64_t begin_ns;
        std::uint64_t end_ns;
        std::span<const std::pair<std::uint32_t, std::uint64_t>> launches;
    };
    using ProfileCallback = void (*)(ProgramError error, std::string_view message,
                                     std::span<const std::byte> readback, const Timestamps& times, void* userdata);
    void run_profiled(const Step& step, std::uint32_t launches, ProfileCallback done, void* userdata);
    [[nodiscard]] std::uint32_t launch_count() const noexcept;
    [[nodiscard]] bool can_profile() const noexcept { return true; }

    // Fires the callbacks of finished steps, oldest first (with `wait`,
    // after blocking until the oldest has finished). Returns how many fired.
    int process_events(bool wait);
    [[nodiscard]] std::uint32_t outstanding() const noexcept;

    ~Program();
    Program(const Program&) = delete;
    Program& operator=(const Program&) = delete;

private:
    Program() = default;
    cb_program* program_ = nullptr;
};

}  // namespace bllm::kernels::cuda
