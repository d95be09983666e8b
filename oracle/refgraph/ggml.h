// Stand-in for the ggml API surface that the reference's decoder, encoder
// and weight loader use (src/motion_dec.cpp, src/motion_enc.cpp,
// src/ops_common.h, src/gguf_load.cpp), so that those files compile where
// they lie and run on the CPU. TEST INFRASTRUCTURE ONLY: the graph these
// files build is evaluated by oracle/refgraph/graph.cpp, whose stock-op
// semantics are restated from ggml's definitions; the patched ops
// (patches/ggml-tp-ops.patch) run the reference's own constructors and CPU
// forward functions, extracted from the patch by oracle/ref_build.py.
// ggml upstream (ggml-org/ggml @ 3af5f576, the reference's absent
// submodule) is not present; nothing here is taken from it.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>

#define GGML_MAX_DIMS 4
#define GGML_MAX_SRC 10
#define GGML_MAX_NAME 64
#define GGML_MAX_OP_PARAMS 64
#define GGML_API

// a failed check raises; the C entry points of the stand-in report it
#define GGML_ASSERT(x)                                                                      \
    do {                                                                                    \
        if (!(x)) throw std::runtime_error(std::string("GGML_ASSERT failed: ") + #x + " (" + \
                                           __FILE__ + ":" + std::to_string(__LINE__) + ")"); \
    } while (0)

enum ggml_type { GGML_TYPE_F32 = 0, GGML_TYPE_F16 = 1 };

enum ggml_op {
    GGML_OP_NONE = 0,
    GGML_OP_DUP,  // cont / cast
    GGML_OP_ADD,
    GGML_OP_MUL,
    GGML_OP_DIV,
    GGML_OP_SQR,
    GGML_OP_SQRT,
    GGML_OP_TANH,
    GGML_OP_SIGMOID,
    GGML_OP_LEAKY_RELU,
    GGML_OP_SCALE_BIAS,
    GGML_OP_CONCAT,
    GGML_OP_REPEAT,
    GGML_OP_MUL_MAT,
    GGML_OP_RESHAPE,
    GGML_OP_VIEW,
    GGML_OP_PERMUTE,
    GGML_OP_IM2COL,
    GGML_OP_CONV_2D,
    GGML_OP_CONV_2D_DW,
    GGML_OP_CONV_TRANSPOSE_2D,
    GGML_OP_UPSCALE,
    GGML_OP_PAD,
    GGML_OP_NORM,
    // the reference's patched ops
    GGML_OP_BILINEAR_GATHER,
    GGML_OP_BIAS_LRELU,
    GGML_OP_SUBPIX_LRELU,
    GGML_OP_SUBPIX_LRELU_CL,
    GGML_OP_UPFIRDN2X,
    GGML_OP_CLSP_MUL,
    GGML_OP_CLSP_LERP,
    GGML_OP_FLOW_GRID,
    GGML_OP_COUNT,
};

enum ggml_scale_mode { GGML_SCALE_MODE_NEAREST = 0, GGML_SCALE_MODE_BILINEAR = 1 };
enum ggml_status { GGML_STATUS_SUCCESS = 0, GGML_STATUS_FAILED = -1 };

typedef uint16_t ggml_fp16_t;

struct ggml_context;
struct ggml_cgraph;

struct ggml_init_params {
    size_t mem_size;
    void *mem_buffer;
    bool no_alloc;
};

enum { GGML_TENSOR_FLAG_INPUT = 1, GGML_TENSOR_FLAG_OUTPUT = 2 };

struct ggml_tensor {
    enum ggml_type type = GGML_TYPE_F32;
    int64_t ne[GGML_MAX_DIMS] = {1, 1, 1, 1};
    size_t nb[GGML_MAX_DIMS] = {0, 0, 0, 0};
    enum ggml_op op = GGML_OP_NONE;
    int32_t op_params[GGML_MAX_OP_PARAMS / sizeof(int32_t)] = {0};
    int32_t flags = 0;
    struct ggml_tensor *src[GGML_MAX_SRC] = {nullptr};
    struct ggml_tensor *view_src = nullptr;
    size_t view_offs = 0;
    void *data = nullptr;
    char name[GGML_MAX_NAME] = {0};
    bool owns_data = false;  // stand-in bookkeeping: data is this tensor's own allocation
};

struct ggml_compute_params {
    int ith = 0;
    int nth = 1;
};

size_t ggml_tensor_overhead(void);
struct ggml_context *ggml_init(struct ggml_init_params params);
void ggml_free(struct ggml_context *ctx);

size_t ggml_type_size(enum ggml_type t);
int64_t ggml_nelements(const struct ggml_tensor *t);
size_t ggml_nbytes(const struct ggml_tensor *t);
bool ggml_is_contiguous(const struct ggml_tensor *t);
bool ggml_are_same_shape(const struct ggml_tensor *a, const struct ggml_tensor *b);
int64_t ggml_calc_conv_output_size(int64_t ins, int64_t ks, int s, int p, int d);

float ggml_fp16_to_fp32(ggml_fp16_t h);
ggml_fp16_t ggml_fp32_to_fp16(float f);
#define GGML_CPU_FP16_TO_FP32(x) ggml_fp16_to_fp32(x)
#define GGML_CPU_FP32_TO_FP16(x) ggml_fp32_to_fp16(x)

struct ggml_tensor *ggml_new_tensor(struct ggml_context *ctx, enum ggml_type type, int n_dims,
                                    const int64_t *ne);
struct ggml_tensor *ggml_new_tensor_1d(struct ggml_context *ctx, enum ggml_type type, int64_t ne0);
struct ggml_tensor *ggml_new_tensor_2d(struct ggml_context *ctx, enum ggml_type type, int64_t ne0,
                                       int64_t ne1);
struct ggml_tensor *ggml_new_tensor_3d(struct ggml_context *ctx, enum ggml_type type, int64_t ne0,
                                       int64_t ne1, int64_t ne2);
struct ggml_tensor *ggml_new_tensor_4d(struct ggml_context *ctx, enum ggml_type type, int64_t ne0,
                                       int64_t ne1, int64_t ne2, int64_t ne3);
struct ggml_tensor *ggml_set_name(struct ggml_tensor *t, const char *name);
void ggml_set_input(struct ggml_tensor *t);
void ggml_set_output(struct ggml_tensor *t);
void ggml_set_op_params(struct ggml_tensor *t, const void *params, size_t size);

// views and layout
struct ggml_tensor *ggml_reshape_2d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1);
struct ggml_tensor *ggml_reshape_3d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1,
                                    int64_t ne2);
struct ggml_tensor *ggml_reshape_4d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1,
                                    int64_t ne2, int64_t ne3);
struct ggml_tensor *ggml_view_2d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1,
                                 size_t nb1, size_t offset);
struct ggml_tensor *ggml_view_3d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1,
                                 int64_t ne2, size_t nb1, size_t nb2, size_t offset);
struct ggml_tensor *ggml_view_4d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1,
                                 int64_t ne2, int64_t ne3, size_t nb1, size_t nb2, size_t nb3, size_t offset);
struct ggml_tensor *ggml_permute(struct ggml_context *ctx, struct ggml_tensor *a, int axis0, int axis1,
                                 int axis2, int axis3);
struct ggml_tensor *ggml_cont(struct ggml_context *ctx, struct ggml_tensor *a);
struct ggml_tensor *ggml_cast(struct ggml_context *ctx, struct ggml_tensor *a, enum ggml_type type);
struct ggml_tensor *ggml_repeat_4d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1,
                                   int64_t ne2, int64_t ne3);
struct ggml_tensor *ggml_concat(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b, int dim);
struct ggml_tensor *ggml_pad_ext(struct ggml_context *ctx, struct ggml_tensor *a, int lp0, int rp0, int lp1,
                                 int rp1, int lp2, int rp2, int lp3, int rp3);
struct ggml_tensor *ggml_upscale(struct ggml_context *ctx, struct ggml_tensor *a, int scale_factor,
                                 enum ggml_scale_mode mode);

// arithmetic
struct ggml_tensor *ggml_add(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b);
struct ggml_tensor *ggml_mul(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b);
struct ggml_tensor *ggml_div(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b);
struct ggml_tensor *ggml_sqr(struct ggml_context *ctx, struct ggml_tensor *a);
struct ggml_tensor *ggml_sqrt(struct ggml_context *ctx, struct ggml_tensor *a);
struct ggml_tensor *ggml_tanh(struct ggml_context *ctx, struct ggml_tensor *a);
struct ggml_tensor *ggml_sigmoid(struct ggml_context *ctx, struct ggml_tensor *a);
struct ggml_tensor *ggml_leaky_relu(struct ggml_context *ctx, struct ggml_tensor *a, float negative_slope,
                                    bool inplace);
struct ggml_tensor *ggml_scale_bias(struct ggml_context *ctx, struct ggml_tensor *a, float s, float b);
struct ggml_tensor *ggml_norm(struct ggml_context *ctx, struct ggml_tensor *a, float eps);
struct ggml_tensor *ggml_mul_mat(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b);

// convolutions
struct ggml_tensor *ggml_im2col(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b, int s0,
                                int s1, int p0, int p1, int d0, int d1, bool is_2D, enum ggml_type dst_type);
struct ggml_tensor *ggml_conv_2d_direct(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b,
                                        int s0, int s1, int p0, int p1, int d0, int d1);
struct ggml_tensor *ggml_conv_2d_dw_direct(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b,
                                           int s0, int s1, int p0, int p1, int d0, int d1);
struct ggml_tensor *ggml_conv_transpose_2d_p0(struct ggml_context *ctx, struct ggml_tensor *a,
                                              struct ggml_tensor *b, int stride);

// the reference's patched ops (constructors extracted from the patch)
struct ggml_tensor *ggml_im2col_cf(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b, int s0,
                                   int s1, int p0, int p1, int d0, int d1, enum ggml_type dst_type);
struct ggml_tensor *ggml_bilinear_gather(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b,
                                         int w, int h);
struct ggml_tensor *ggml_bilinear_gather_sp(struct ggml_context *ctx, struct ggml_tensor *a,
                                            struct ggml_tensor *b, int w, int h);
struct ggml_tensor *ggml_bilinear_gather_planar(struct ggml_context *ctx, struct ggml_tensor *a,
                                                struct ggml_tensor *b, int w, int h);
struct ggml_tensor *ggml_bias_lrelu(struct ggml_context *ctx, struct ggml_tensor *x, struct ggml_tensor *bias,
                                    int axis, float slope);
struct ggml_tensor *ggml_subpix_lrelu(struct ggml_context *ctx, struct ggml_tensor *g0, struct ggml_tensor *g1,
                                      struct ggml_tensor *bias, float slope);
struct ggml_tensor *ggml_subpix_lrelu_cl(struct ggml_context *ctx, struct ggml_tensor *y4,
                                         struct ggml_tensor *bias, int w, float slope);
struct ggml_tensor *ggml_flow_grid(struct ggml_context *ctx, struct ggml_tensor *fl, struct ggml_tensor *xs);
struct ggml_tensor *ggml_clsp_mul(struct ggml_context *ctx, struct ggml_tensor *cl, struct ggml_tensor *m);
struct ggml_tensor *ggml_clsp_lerp(struct ggml_context *ctx, struct ggml_tensor *cl, struct ggml_tensor *m,
                                   struct ggml_tensor *out_sp);
struct ggml_tensor *ggml_upfirdn2x(struct ggml_context *ctx, struct ggml_tensor *x, struct ggml_tensor *kern);

// graphs
struct ggml_cgraph *ggml_new_graph_custom(struct ggml_context *ctx, size_t size, bool grads);
void ggml_build_forward_expand(struct ggml_cgraph *gf, struct ggml_tensor *t);
int ggml_graph_n_nodes(struct ggml_cgraph *gf);
struct ggml_tensor *ggml_graph_node(struct ggml_cgraph *gf, int i);
