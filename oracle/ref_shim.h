// Minimal stand-ins that let the reference's own op code, extracted verbatim
// from patches/ggml-tp-ops.patch by oracle/ref_build.py, compile as plain host
// C++ into oracle/_ref/. TEST INFRASTRUCTURE ONLY: the result is the
// reference-side pin for the oracle's op restatements.
//
// Two families are covered:
//   * the patch's ggml CPU forward functions (need ggml_tensor,
//     ggml_compute_params and the fp16 helpers);
//   * the patch's CUDA kernels (need __global__, half and the
//     blockIdx/threadIdx/blockDim builtins, which are emulated here by looping
//     one host thread over every (block, thread) pair).
#pragma once

#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstring>

// ---- ggml CPU side -------------------------------------------------------
enum ggml_type { GGML_TYPE_F32 = 0, GGML_TYPE_F16 = 1 };
typedef uint16_t ggml_fp16_t;

struct ggml_tensor {
    ggml_type type = GGML_TYPE_F32;
    int64_t ne[4] = {1, 1, 1, 1};
    size_t nb[4] = {0, 0, 0, 0};
    int32_t op_params[16] = {0};
    ggml_tensor *src[10] = {nullptr};
    void *data = nullptr;
};
struct ggml_compute_params {
    int ith = 0;
    int nth = 1;
};
static inline int64_t ggml_nelements(const ggml_tensor *t) {
    return t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3];
}
static inline float GGML_CPU_FP16_TO_FP32(ggml_fp16_t h) {
    _Float16 v;
    memcpy(&v, &h, 2);
    return (float) v;
}

// ---- CUDA kernel side ----------------------------------------------------
#define __global__
struct ref_dim3 {
    unsigned x = 0, y = 0, z = 0;
};
extern thread_local ref_dim3 blockIdx, threadIdx, blockDim;

struct half {
    uint16_t bits;
    operator float() const {
        _Float16 v;
        memcpy(&v, &bits, 2);
        return (float) v;
    }
    half &operator=(float f) {
        _Float16 v = (_Float16) f;
        memcpy(&bits, &v, 2);
        return *this;
    }
};
