// C ABI entry points: argument checks, dispatch to the kernels, status codes.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "api_common.h"
#include "charlotte_b200.h"
#include "matmul.h"
#include "tma.cuh"

namespace cb {

namespace {
thread_local std::string g_error;
// Two words a device: [0] set by a kernel whose bounded wait ran out; [1]
// 1 + the polls of a first wait on a copy when a test shortened them
// (cb_debug_spin_limit), else 0.
__device__ unsigned int g_fault_word[2];
}

int fail(int status, const char* format, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, format);
    vsnprintf(buf, sizeof buf, format, ap);
    va_end(ap);
    g_error = buf;
    return status;
}

int fail_cuda(cudaError_t e, const char* what) {
    // Errors that leave the context unusable (sticky) are the device lost.
    const bool sticky = e == cudaErrorIllegalAddress || e == cudaErrorLaunchFailure ||
                        e == cudaErrorIllegalInstruction || e == cudaErrorMisalignedAddress ||
                        e == cudaErrorHardwareStackError || e == cudaErrorAssert ||
                        e == cudaErrorDevicesUnavailable || e == cudaErrorECCUncorrectable;
    return fail(sticky ? CB_ERROR_DEVICE_LOST : CB_ERROR_STEP, "%s: %s (%s)", what, cudaGetErrorString(e),
                cudaGetErrorName(e));
}

int sm_count() {
    static int counts[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
    if (counts[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
        counts[dev] = n;
    }
    return counts[dev];
}

unsigned int* fault_word() {
    static unsigned int* words[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    if (!words[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_fault_word) != cudaSuccess) return nullptr;
        words[dev] = static_cast<unsigned int*>(p);
    }
    return words[dev];
}

}  // namespace cb

extern "C" {

int cb_debug_spin_limit(int32_t polls) {
    unsigned int* w = cb::fault_word();
    if (!w) return cb::fail(CB_ERROR_STEP, "cb_debug_spin_limit: no CUDA device");
    if (polls >= static_cast<int32_t>(cb::kSpinLimit)) polls = -1;
    const uint32_t word = polls < 0 ? 0u : static_cast<uint32_t>(polls) + 1u;
    const cudaError_t e = cudaMemcpy(w + 1, &word, sizeof word, cudaMemcpyHostToDevice);
    return e == cudaSuccess ? CB_OK : cb::fail_cuda(e, "cb_debug_spin_limit");
}

int cb_fault_check(unsigned int* faults) {
    unsigned int* w = cb::fault_word();
    if (!w) return cb::fail(CB_ERROR_STEP, "cb_fault_check: no CUDA device");
    unsigned int h = 0;
    cudaError_t e = cudaMemcpy(&h, w, sizeof h, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cb::fail_cuda(e, "cb_fault_check");
    if (h) {
        const unsigned int zero = 0;
        e = cudaMemcpy(w, &zero, sizeof zero, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return cb::fail_cuda(e, "cb_fault_check");
    }
    if (faults) *faults = h;
    return h ? cb::fail(CB_ERROR_STEP, "a kernel's bounded wait ran out (fault word 0x%x)", h) : CB_OK;
}


size_t cb_last_error(char* buffer, size_t capacity) {
    const std::string& e = cb::g_error;
    if (buffer && capacity) {
        const size_t n = e.size() < capacity - 1 ? e.size() : capacity - 1;
        std::memcpy(buffer, e.data(), n);
        buffer[n] = '\0';
    }
    return e.size();
}

const char* cb_version(void) { return "0.1.0"; }

int cb_device_sm_count(void) {
    const int n = cb::sm_count();
    return n > 0 ? n : cb::fail(CB_ERROR_STEP, "no CUDA device");
}

uint64_t cb_matmul_split_bytes(uint32_t tokens, uint32_t rows) {
    return 32ull * tokens * rows * sizeof(float);
}

uint64_t cb_matmul_scratch_bytes(uint32_t flags, uint32_t tokens, uint32_t columns) {
    return (flags & CB_MATMUL_TENSOR) ? cb::matmul_tensor_scratch_bytes(tokens, columns) : 0u;
}

namespace {

// The product's description checked and copied into `a` (members, rows,
// epilogue); `who` names the entry point in messages.
int product_of(const cb_matmul* m, cb::MatmulArgs& a, const char* who) {
    using namespace cb;
    if (!m) return fail(CB_ERROR_INVALID, "%s: null argument", who);
    if (m->format != CB_Q4_0 && m->format != CB_Q4_1 && m->format != CB_Q8_0 && m->format != CB_Q6_K &&
        m->format != CB_BF16)
        return fail(CB_ERROR_INVALID, "%s: format %u has no matmul kernel", who, m->format);
    if (m->columns == 0 || m->columns % 32 != 0)
        return fail(CB_ERROR_INVALID, "%s: columns %u is not a whole number of 32-weight groups", who, m->columns);
    if (m->format == CB_Q6_K && m->columns % 256 != 0)
        return fail(CB_ERROR_INVALID, "%s: Q6_K rows of %u are not whole 256-weight super-blocks", who, m->columns);
    if (m->members < 1 || m->members > 3) return fail(CB_ERROR_INVALID, "%s: %u members", who, m->members);
    if (m->epilogue > CB_EPILOGUE_GATED_BY_INPUT) return fail(CB_ERROR_INVALID, "%s: epilogue %u", who, m->epilogue);
    if (m->activation > CB_ACT_SIGMOID) return fail(CB_ERROR_INVALID, "%s: activation %u", who, m->activation);
    if (m->epilogue == CB_EPILOGUE_GATED && (m->members != 2 || m->member[0].rows != m->member[1].rows))
        return fail(CB_ERROR_INVALID, "%s: a gated product is a gate and an up of equal rows", who);
    a.format = m->format;
    a.columns = m->columns;
    a.members = m->members;
    a.epilogue = m->epilogue;
    a.activation = m->activation;
    uint32_t total = 0;
    for (uint32_t i = 0; i < m->members; ++i) {
        const cb_member& s = m->member[i];
        if (!s.piece || !aligned16(s.piece))
            return fail(CB_ERROR_INVALID, "%s: member %u's piece is null or not 16-byte aligned", who, i);
        if (s.rows == 0) return fail(CB_ERROR_INVALID, "%s: member %u has no rows", who, i);
        const uint64_t groups = static_cast<uint64_t>(s.first_row + s.rows) * (m->columns / 32);
        // stored blocks: a Q6_K super-block holds 8 groups, a BF16 block one value
        const uint64_t needed_blocks = m->format == CB_Q6_K ? groups / 8 : (m->format == CB_BF16 ? groups * 32 : groups);
        if (needed_blocks > s.blocks)
            return fail(CB_ERROR_INVALID, "%s: member %u reads rows past its piece (%llu of %u blocks)", who, i,
                        static_cast<unsigned long long>(needed_blocks), s.blocks);
        a.member[i] = {static_cast<const uint8_t*>(s.piece), s.blocks, s.first_row, s.rows, s.out_offset};
        total += s.rows;
    }
    a.total_rows = m->epilogue == CB_EPILOGUE_GATED ? m->member[0].rows : total;
    return CB_OK;
}

}  // namespace

uint64_t cb_matmul_dense_bytes(const cb_matmul* m) {
    cb::MatmulArgs a{};
    if (product_of(m, a, "cb_matmul_dense_bytes") != CB_OK) return 0;
    return cb::matmul_dense_bytes(a);
}

int cb_matmul_densify(const cb_matmul* m, void* dense, uint64_t dense_bytes, void* stream) {
    using namespace cb;
    MatmulArgs a{};
    if (int rc = product_of(m, a, "cb_matmul_densify")) return rc;
    if (!dense || !aligned16(dense) || dense_bytes < matmul_dense_bytes(a))
        return fail(CB_ERROR_INVALID, "cb_matmul_densify: needs %llu bytes of 16-byte aligned memory",
                    static_cast<unsigned long long>(matmul_dense_bytes(a)));
    if (cudaError_t e = matmul_densify(a, dense, static_cast<cudaStream_t>(stream)); e != cudaSuccess)
        return fail_cuda(e, "cb_matmul_densify: launch");
    return CB_OK;
}

int cb_matmul_run(const cb_matmul* m, const float* x, uint32_t x_stride, uint32_t tokens, float* const out[3],
                  const uint32_t out_stride[3], uint32_t flags, void* stream) {
    using namespace cb;
    if (!m || !x || !out) return fail(CB_ERROR_INVALID, "cb_matmul_run: null argument");
    MatmulArgs a{};
    if (int rc = product_of(m, a, "cb_matmul_run")) return rc;
    if (m->epilogue == CB_EPILOGUE_GATED_BY_INPUT && !m->gate_input)
        return fail(CB_ERROR_INVALID, "cb_matmul_run: GATED_BY_INPUT without its input u");
    if (tokens == 0) return CB_OK;
    if (x_stride < m->columns) return fail(CB_ERROR_INVALID, "cb_matmul_run: x_stride %u < columns", x_stride);
    if (!aligned16(x) || x_stride % 4 != 0)
        return fail(CB_ERROR_INVALID, "cb_matmul_run: x must be 16-byte aligned with a stride of whole float4s");
    a.token = m->gate_input_token;
    a.tokens = tokens;
    a.x = x;
    a.x_stride = x_stride;
    a.gate_input = m->gate_input;
    a.gate_input_stride = m->gate_input_stride;
    a.gate_input_column = m->gate_input_column;
    a.fault = fault_word();
    if (matmul_decode_smem_bytes(m->format, m->columns) > 220u * 1024u)
        return fail(CB_ERROR_INVALID, "cb_matmul_run: rows of %u are wider than the decode form stages", m->columns);
    const uint32_t total = m->epilogue == CB_EPILOGUE_GATED ? 2 * m->member[0].rows : a.total_rows;
    const uint32_t outputs = m->epilogue == CB_EPILOGUE_QKV ? m->members : 1;
    for (uint32_t i = 0; i < outputs; ++i) {
        if (!out[i]) return fail(CB_ERROR_INVALID, "cb_matmul_run: output %u is null", i);
        a.out[i] = out[i];
        a.out_stride[i] = out_stride ? out_stride[i] : 0;
        if (tokens > 1 && a.out_stride[i] == 0)
            return fail(CB_ERROR_INVALID, "cb_matmul_run: output %u has no stride for %u tokens", i, tokens);
    }
    if (flags & CB_MATMUL_TENSOR) {
        const uint64_t need = matmul_tensor_scratch_bytes(tokens, m->columns);
        if (!m->scratch || !aligned16(m->scratch) || m->scratch_bytes < need)
            return fail(CB_ERROR_INVALID, "cb_matmul_run: the tensor form needs %llu bytes of 16-byte aligned scratch",
                        static_cast<unsigned long long>(need));
        a.scratch = m->scratch;
        a.scratch_bytes = m->scratch_bytes;
        if (m->dense) {
            if (!aligned16(m->dense))
                return fail(CB_ERROR_INVALID, "cb_matmul_run: the dense weights must be 16-byte aligned");
            a.dense = m->dense;
            if (m->x16 && !aligned16(m->x16))
                return fail(CB_ERROR_INVALID, "cb_matmul_run: x16 must be 16-byte aligned");
            if (m->out16 && m->epilogue != CB_EPILOGUE_GATED)
                return fail(CB_ERROR_INVALID, "cb_matmul_run: out16 is the gated epilogue's");
            a.x16 = m->x16;
            a.out16 = m->out16;
        } else if (m->x16 || m->out16) {
            return fail(CB_ERROR_INVALID, "cb_matmul_run: x16 and out16 are the dense form's");
        }
    }
    const int sms = sm_count();
    if (sms <= 0) return fail(CB_ERROR_STEP, "cb_matmul_run: no CUDA device");
    const bool pdl = (flags & CB_MATMUL_PDL) != 0;
    const uint32_t slots = total;
    bool tiled = tiled_form(tokens, slots);
    if (flags & CB_MATMUL_STREAMED) tiled = false;
    if (flags & CB_MATMUL_TILED) tiled = true;
    // The split form: asked for, or chosen for a few-tile product when the
    // caller gave range-sum scratch and no other form.
    const uint64_t split_need = cb_matmul_split_bytes(tokens, total);
    const bool split_scratch = m->scratch && aligned16(m->scratch) && m->scratch_bytes >= split_need;
    bool split = (flags & CB_MATMUL_SPLIT) != 0;
    if (split && (m->epilogue == CB_EPILOGUE_GATED || !split_scratch || (flags & CB_MATMUL_TENSOR)))
        return fail(CB_ERROR_INVALID, "cb_matmul_run: the split form takes no gated product and needs %llu bytes of "
                    "16-byte aligned range-sum scratch", static_cast<unsigned long long>(split_need));
    if (!split && split_scratch && tokens > 1 &&
        !(flags & (CB_MATMUL_TENSOR | CB_MATMUL_STREAMED | CB_MATMUL_TILED)) &&
        split_form(tokens, slots, m->columns, m->epilogue, sms))
        split = true;
    if (split) a.range_sums = static_cast<float*>(m->scratch);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = (flags & CB_MATMUL_TENSOR) ? (a.dense ? matmul_dense(a, sms, st, pdl) : matmul_tensor(a, st, pdl))
                    : split                    ? matmul_split(a, sms, st, pdl)
                    : tiled                    ? matmul_tiled(a, sms, st, pdl)
                                               : matmul_decode(a, sms, st, pdl);
    if (e != cudaSuccess) return fail_cuda(e, "cb_matmul_run: launch");
    return CB_OK;
}

}  // extern "C"
