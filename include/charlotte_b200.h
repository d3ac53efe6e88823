/*
 * charlotte_b200 — the C ABI of a B200 (sm_100a) CUDA backend for the hot
 * path of Charlotte (plainsight-systems/charlotte): GGUF dequant-matmul over
 * Q4_0 / Q8_0 / repacked Q6_K, RMSNorm, QK-norm + RoPE + KV append, chunked
 * attention over the f16 KV cache, embedding gather, top-k selection and the
 * draw. It stands where the reference's WebGPU dispatch layer
 * (src/core/kernels/program.{h,cpp}) and its WGSL kernels stand; the
 * reference's launchers, graph, KV-cache bookkeeping and loader are unchanged
 * callers.
 *
 * Conventions. Plain pointers and sizes only. Every buffer argument is a CUDA
 * device pointer unless its name says `host`. A `stream` is a cudaStream_t
 * (NULL: the legacy default stream). Weight pieces are in the reference's
 * device layout (src/core/formats/device_layout.h:121-136), each piece's
 * first byte 16-byte aligned and its length padded to 16. Every function
 * returns a cb_status; on failure cb_last_error() gives the calling thread's
 * message. Nothing here traps or spins without bound: a failed launch or an
 * invalid argument is a status, never a fault on purpose.
 */
#ifndef CHARLOTTE_B200_H
#define CHARLOTTE_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define CB_API __attribute__((visibility("default")))
#else
#define CB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* The five meanings of the reference's ProgramError
 * (src/core/kernels/program.h:71-77), plus argument errors. */
typedef enum cb_status {
    CB_OK = 0,
    CB_ERROR_BUILD = 1,        /* a program could not be built */
    CB_ERROR_STEP = 2,         /* a step (or a kernel call) failed to run */
    CB_ERROR_DEVICE_LOST = 3,  /* the CUDA context is no longer usable */
    CB_ERROR_CANCELLED = 4,    /* a step refused or abandoned unrun */
    CB_ERROR_INVALID = 5       /* an argument broke a stated precondition */
} cb_status;

/* GGUF tensor types a weight may take (src/core/gguf/types.h:41-43). */
enum { CB_F32 = 0, CB_F16 = 1, CB_Q4_0 = 2, CB_Q8_0 = 8, CB_Q6_K = 14 };

/* Copies the calling thread's last error message (NUL-terminated, truncated
 * to `capacity`); returns its full length. Replaces the message the
 * reference's callbacks carry (program.h:159-169). */
CB_API size_t cb_last_error(char* buffer, size_t capacity);

/* The library's version, "major.minor.patch". */
CB_API const char* cb_version(void);

/* The current device's streaming multiprocessor count (148 on a B200), or
 * a negative status. */
CB_API int cb_device_sm_count(void);

/* Reads and clears the current device's fault word: kernels whose bounded
 * waits ran out (a copy or a peer that never arrived) set bits in it instead
 * of spinning forever. Synchronizes the device. CB_OK when no bit was set;
 * otherwise CB_ERROR_STEP, with the bits in *faults (may be NULL). */
CB_API int cb_fault_check(unsigned int* faults);

/* ---- matrix products --------------------------------------------------------
 * Replaces the matmul kernel's entry points decode_write, decode_qkv,
 * decode_gated, decode_gated_input (src/core/kernels/matmul/matmul.wgsl
 * :287-361) and the prefill forms (:520-695) behind matmul_launches
 * (src/core/kernels/matmul/matmul.h:672). One member is one weight piece;
 * a fused group (Q,K,V or gate,up) is two or three members, as the
 * reference's Matmul constants (matmul.wgsl:28-40) describe them. */
enum {
    CB_EPILOGUE_WRITE = 0,           /* y to out[0]                                  */
    CB_EPILOGUE_QKV = 1,             /* member m's rows to out[m]                     */
    CB_EPILOGUE_GATED = 2,           /* act(gate)·up to out[0]; members gate, up      */
    CB_EPILOGUE_GATED_BY_INPUT = 3   /* act(y)·u[t·stride + column + o] to out[0]     */
};
enum { CB_ACT_SILU = 0, CB_ACT_GELU_TANH = 1, CB_ACT_SIGMOID = 2 };

/* Flags of cb_matmul_run. */
enum {
    CB_MATMUL_PDL = 1u,      /* launch with programmatic dependent launch   */
    CB_MATMUL_TENSOR = 2u    /* tokens > 1: the tcgen05 tensor-core form     */
};

typedef struct cb_member {
    const void* piece;     /* the weight piece (device layout), 16-B aligned          */
    uint32_t blocks;       /* blocks in the piece: locates each of its streams        */
    uint32_t first_row;    /* first weight row read (a GLU half's first row; else 0)  */
    uint32_t rows;         /* rows this member gives the product                      */
    uint32_t out_offset;   /* Write: first output column of its rows; otherwise 0     */
} cb_member;

typedef struct cb_matmul {
    uint32_t format;               /* CB_Q4_0, CB_Q8_0 or CB_Q6_K                        */
    uint32_t columns;              /* K, a multiple of 32                                */
    uint32_t members;              /* 1 to 3                                             */
    uint32_t epilogue;             /* CB_EPILOGUE_*                                      */
    uint32_t activation;           /* CB_ACT_*: GATED and GATED_BY_INPUT                 */
    cb_member member[3];
    const float* gate_input;       /* GATED_BY_INPUT's u, else NULL                      */
    uint32_t gate_input_stride;    /* floats between u's token rows                      */
    uint32_t gate_input_column;    /* u's first column                                   */
    uint32_t gate_input_token;     /* u's row of the first token                         */
} cb_matmul;

/* y[t][o] = Σ_k W[o][k]·x[t][k] for tokens t in [0, tokens), each output
 * added in the reference's order (matmul.h:34-50) unless CB_MATMUL_TENSOR.
 * x: [tokens][x_stride] f32. out[m]: [tokens][out_stride[m]] f32 (unused
 * entries may be NULL). */
CB_API int cb_matmul_run(const cb_matmul* m, const float* x, uint32_t x_stride, uint32_t tokens, float* const out[3],
                  const uint32_t out_stride[3], uint32_t flags, void* stream);

#ifdef __cplusplus
}
#endif
#endif
