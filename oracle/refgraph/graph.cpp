// Eager evaluator behind the ggml stand-in (ggml.h), plus the pieces of the
// reference's runtime glue that its decoder and encoder need (plan_t, the
// tap sink, read_file, linear; restated from src/backend.cpp:68-189,
// 193-246 and src/dump.cpp in this file's own form). TEST INFRASTRUCTURE
// ONLY: it exists so that the reference's own src/motion_dec.cpp,
// src/motion_enc.cpp and src/gguf_load.cpp run on the CPU and pin the oracle
// at graph level (oracle/ref_build.py compiles them from where they lie).
//
// Graph model: op constructors record nodes (type, shape, strides, sources,
// parameters); views, reshapes and permutes alias their source's storage.
// plan_t::compute evaluates the nodes of its graph in topological order,
// allocating each result when it is computed and freeing it after its last
// consumer (outputs stay until the next compute).
//
// Stock-op semantics, restated from ggml's definitions:
//   add/mul/div  dst[i] = a[i] op b[i mod b.ne] (b repeats over a), dst type = a's
//   mul_mat      dst[m, n, i2, i3] = sum_k a[k, m, i2/r2, i3/r3] * b[k, n, i2, i3], F32;
//                an F16 `a` makes b round to F16 first (the CPU backend's
//                vec_dot type for F16 weights)
//   conv_2d_direct  a [KW,KH,IC,OC], b [W,H,IC,N] -> [OW,OH,OC,N] (cross-correlation);
//                an F16 kernel rounds the input to F16
//   conv_2d_dw_direct  a [KW,KH,1,C]: per-channel cross-correlation
//   conv_transpose_2d_p0  a [KW,KH,OC,IC]: dst[x*s+kx, y*s+ky, oc] += a[kx,ky,oc,ic] b[x,y,ic]
//   im2col       [IC*KH*KW, OW, OH, N], row iic*KH*KW + ikh*KW + ikw; the patch's
//                channels-first flag (op_params[6] bit 1) takes [IC, IW, IH, N] and rows
//                ic + IC*(kw + KW*kh) (patch:201-307)
//   pad_ext (zeros), upscale (nearest, integer factor), concat, repeat_4d,
//   cont, cast (round to nearest even), sqr, sqrt, tanh, sigmoid
//   1/(1+exp(-x)), leaky_relu, scale_bias a*s+b.
#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <map>
#include <memory>
#include <set>
#include <unordered_map>
#include <vector>

#include "ggml-alloc.h"
#include "ggml-backend.h"
#include "tp_internal.h"
#include "dump_standin.h"

// the patch's CPU forward functions (extracted by oracle/ref_build.py)
void ggml_compute_forward_bilinear_gather(const ggml_compute_params *params, ggml_tensor *dst);
void ggml_compute_forward_bias_lrelu(const ggml_compute_params *params, ggml_tensor *dst);
void ggml_compute_forward_subpix_lrelu(const ggml_compute_params *params, ggml_tensor *dst);
void ggml_compute_forward_subpix_lrelu_cl(const ggml_compute_params *params, ggml_tensor *dst);
void ggml_compute_forward_upfirdn2x(const ggml_compute_params *params, ggml_tensor *dst);
void ggml_compute_forward_clsp_mul(const ggml_compute_params *params, ggml_tensor *dst);
void ggml_compute_forward_clsp_lerp(const ggml_compute_params *params, ggml_tensor *dst);
void ggml_compute_forward_flow_grid(const ggml_compute_params *params, ggml_tensor *dst);

struct ggml_context {
    bool no_alloc = true;
    std::vector<std::unique_ptr<ggml_tensor>> tensors;
    std::vector<std::unique_ptr<ggml_cgraph>> graphs;
};

struct ggml_cgraph {
    std::vector<ggml_tensor *> nodes;
    std::set<const ggml_tensor *> seen;
};

struct ggml_backend_buffer {
    std::vector<ggml_tensor *> owned;
};

// ---------------------------------------------------------------------------
// basics
// ---------------------------------------------------------------------------
size_t ggml_tensor_overhead(void) { return 512; }

ggml_context *ggml_init(ggml_init_params p) {
    ggml_context *c = new ggml_context();
    c->no_alloc = p.no_alloc;
    return c;
}

static void free_data(ggml_tensor *t) {
    if (t->owns_data) free(t->data);
    t->owns_data = false;
    t->data = nullptr;
}

void ggml_free(ggml_context *ctx) {
    if (!ctx) return;
    for (auto &t : ctx->tensors) free_data(t.get());
    delete ctx;
}

size_t ggml_type_size(ggml_type t) { return t == GGML_TYPE_F16 ? 2 : 4; }
int64_t ggml_nelements(const ggml_tensor *t) { return t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3]; }
size_t ggml_nbytes(const ggml_tensor *t) {
    size_t n = ggml_type_size(t->type);
    for (int i = 0; i < 4; i++) n += (size_t) (t->ne[i] - 1) * t->nb[i];
    return n;
}
bool ggml_is_contiguous(const ggml_tensor *t) {
    size_t s = ggml_type_size(t->type);
    for (int i = 0; i < 4; i++) {
        if (t->ne[i] != 1 && t->nb[i] != s) return false;
        s *= (size_t) t->ne[i];
    }
    return true;
}
bool ggml_are_same_shape(const ggml_tensor *a, const ggml_tensor *b) {
    for (int i = 0; i < 4; i++)
        if (a->ne[i] != b->ne[i]) return false;
    return true;
}
int64_t ggml_calc_conv_output_size(int64_t ins, int64_t ks, int s, int p, int d) {
    return (ins + 2 * p - d * (ks - 1) - 1) / s + 1;
}

float ggml_fp16_to_fp32(ggml_fp16_t h) {
    _Float16 v;
    memcpy(&v, &h, 2);
    return (float) v;
}
ggml_fp16_t ggml_fp32_to_fp16(float f) {
    const _Float16 v = (_Float16) f;  // round to nearest even
    ggml_fp16_t h;
    memcpy(&h, &v, 2);
    return h;
}
static inline float round_f16(float f) { return (float) (_Float16) f; }

static void set_contiguous_strides(ggml_tensor *t) {
    t->nb[0] = ggml_type_size(t->type);
    for (int i = 1; i < 4; i++) t->nb[i] = t->nb[i - 1] * (size_t) t->ne[i - 1];
}

static ggml_tensor *new_tensor(ggml_context *ctx, ggml_type type, const int64_t ne[4]) {
    auto t = std::make_unique<ggml_tensor>();
    t->type = type;
    for (int i = 0; i < 4; i++) t->ne[i] = ne[i];
    set_contiguous_strides(t.get());
    if (!ctx->no_alloc) {
        t->data = calloc(1, ggml_nbytes(t.get()));
        t->owns_data = true;
    }
    ctx->tensors.push_back(std::move(t));
    return ctx->tensors.back().get();
}

ggml_tensor *ggml_new_tensor(ggml_context *ctx, ggml_type type, int n_dims, const int64_t *ne) {
    int64_t n[4] = {1, 1, 1, 1};
    for (int i = 0; i < n_dims && i < 4; i++) n[i] = ne[i];
    return new_tensor(ctx, type, n);
}
ggml_tensor *ggml_new_tensor_1d(ggml_context *ctx, ggml_type type, int64_t ne0) {
    const int64_t n[4] = {ne0, 1, 1, 1};
    return new_tensor(ctx, type, n);
}
ggml_tensor *ggml_new_tensor_2d(ggml_context *ctx, ggml_type type, int64_t ne0, int64_t ne1) {
    const int64_t n[4] = {ne0, ne1, 1, 1};
    return new_tensor(ctx, type, n);
}
ggml_tensor *ggml_new_tensor_3d(ggml_context *ctx, ggml_type type, int64_t ne0, int64_t ne1, int64_t ne2) {
    const int64_t n[4] = {ne0, ne1, ne2, 1};
    return new_tensor(ctx, type, n);
}
ggml_tensor *ggml_new_tensor_4d(ggml_context *ctx, ggml_type type, int64_t ne0, int64_t ne1, int64_t ne2,
                                int64_t ne3) {
    const int64_t n[4] = {ne0, ne1, ne2, ne3};
    return new_tensor(ctx, type, n);
}
ggml_tensor *ggml_set_name(ggml_tensor *t, const char *name) {
    snprintf(t->name, sizeof t->name, "%s", name);
    return t;
}
void ggml_set_input(ggml_tensor *t) { t->flags |= GGML_TENSOR_FLAG_INPUT; }
void ggml_set_output(ggml_tensor *t) { t->flags |= GGML_TENSOR_FLAG_OUTPUT; }
void ggml_set_op_params(ggml_tensor *t, const void *params, size_t size) {
    GGML_ASSERT(size <= sizeof t->op_params);
    memcpy(t->op_params, params, size);
}

// a node of the given op computing from sources (contiguous result)
static ggml_tensor *node(ggml_context *ctx, ggml_op op, ggml_type type, const int64_t ne[4], ggml_tensor *a,
                         ggml_tensor *b = nullptr, ggml_tensor *c = nullptr) {
    ggml_tensor *t = new_tensor(ctx, type, ne);
    t->op = op;
    t->src[0] = a;
    t->src[1] = b;
    t->src[2] = c;
    return t;
}

// an alias of a's storage with its own shape and strides
static ggml_tensor *alias(ggml_context *ctx, ggml_op op, ggml_tensor *a, const int64_t ne[4], const size_t nb[4],
                          size_t offs) {
    auto t = std::make_unique<ggml_tensor>();
    t->type = a->type;
    for (int i = 0; i < 4; i++) {
        t->ne[i] = ne[i];
        t->nb[i] = nb[i];
    }
    t->op = op;
    t->src[0] = a;
    t->view_src = a;
    t->view_offs = offs;
    if (a->data) t->data = (char *) a->data + offs;
    ctx->tensors.push_back(std::move(t));
    return ctx->tensors.back().get();
}

// ---------------------------------------------------------------------------
// views and layout
// ---------------------------------------------------------------------------
static ggml_tensor *reshape(ggml_context *ctx, ggml_tensor *a, int64_t n0, int64_t n1, int64_t n2, int64_t n3) {
    GGML_ASSERT(ggml_is_contiguous(a));
    GGML_ASSERT(n0 * n1 * n2 * n3 == ggml_nelements(a));
    const int64_t ne[4] = {n0, n1, n2, n3};
    size_t nb[4];
    nb[0] = ggml_type_size(a->type);
    for (int i = 1; i < 4; i++) nb[i] = nb[i - 1] * (size_t) ne[i - 1];
    return alias(ctx, GGML_OP_RESHAPE, a, ne, nb, 0);
}
ggml_tensor *ggml_reshape_2d(ggml_context *ctx, ggml_tensor *a, int64_t ne0, int64_t ne1) {
    return reshape(ctx, a, ne0, ne1, 1, 1);
}
ggml_tensor *ggml_reshape_3d(ggml_context *ctx, ggml_tensor *a, int64_t ne0, int64_t ne1, int64_t ne2) {
    return reshape(ctx, a, ne0, ne1, ne2, 1);
}
ggml_tensor *ggml_reshape_4d(ggml_context *ctx, ggml_tensor *a, int64_t ne0, int64_t ne1, int64_t ne2,
                             int64_t ne3) {
    return reshape(ctx, a, ne0, ne1, ne2, ne3);
}
ggml_tensor *ggml_view_2d(ggml_context *ctx, ggml_tensor *a, int64_t ne0, int64_t ne1, size_t nb1, size_t offset) {
    const int64_t ne[4] = {ne0, ne1, 1, 1};
    const size_t nb[4] = {a->nb[0], nb1, nb1 * (size_t) ne1, nb1 * (size_t) ne1};
    return alias(ctx, GGML_OP_VIEW, a, ne, nb, offset);
}
ggml_tensor *ggml_view_3d(ggml_context *ctx, ggml_tensor *a, int64_t ne0, int64_t ne1, int64_t ne2, size_t nb1,
                          size_t nb2, size_t offset) {
    const int64_t ne[4] = {ne0, ne1, ne2, 1};
    const size_t nb[4] = {a->nb[0], nb1, nb2, nb2 * (size_t) ne2};
    return alias(ctx, GGML_OP_VIEW, a, ne, nb, offset);
}
ggml_tensor *ggml_view_4d(ggml_context *ctx, ggml_tensor *a, int64_t ne0, int64_t ne1, int64_t ne2, int64_t ne3,
                          size_t nb1, size_t nb2, size_t nb3, size_t offset) {
    const int64_t ne[4] = {ne0, ne1, ne2, ne3};
    const size_t nb[4] = {a->nb[0], nb1, nb2, nb3};
    return alias(ctx, GGML_OP_VIEW, a, ne, nb, offset);
}
ggml_tensor *ggml_permute(ggml_context *ctx, ggml_tensor *a, int axis0, int axis1, int axis2, int axis3) {
    const int ax[4] = {axis0, axis1, axis2, axis3};
    int64_t ne[4];
    size_t nb[4];
    for (int i = 0; i < 4; i++) {
        GGML_ASSERT(ax[i] >= 0 && ax[i] < 4);
        ne[ax[i]] = a->ne[i];
        nb[ax[i]] = a->nb[i];
    }
    return alias(ctx, GGML_OP_PERMUTE, a, ne, nb, 0);
}
ggml_tensor *ggml_cont(ggml_context *ctx, ggml_tensor *a) { return node(ctx, GGML_OP_DUP, a->type, a->ne, a); }
ggml_tensor *ggml_cast(ggml_context *ctx, ggml_tensor *a, ggml_type type) {
    return node(ctx, GGML_OP_DUP, type, a->ne, a);
}
ggml_tensor *ggml_repeat_4d(ggml_context *ctx, ggml_tensor *a, int64_t ne0, int64_t ne1, int64_t ne2,
                            int64_t ne3) {
    const int64_t ne[4] = {ne0, ne1, ne2, ne3};
    for (int i = 0; i < 4; i++) GGML_ASSERT(ne[i] % a->ne[i] == 0);
    return node(ctx, GGML_OP_REPEAT, a->type, ne, a);
}
ggml_tensor *ggml_concat(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b, int dim) {
    GGML_ASSERT(dim >= 0 && dim < 4 && a->type == b->type);
    int64_t ne[4];
    for (int i = 0; i < 4; i++) {
        if (i != dim) GGML_ASSERT(a->ne[i] == b->ne[i]);
        ne[i] = i == dim ? a->ne[i] + b->ne[i] : a->ne[i];
    }
    ggml_tensor *t = node(ctx, GGML_OP_CONCAT, a->type, ne, a, b);
    t->op_params[0] = dim;
    return t;
}
ggml_tensor *ggml_pad_ext(ggml_context *ctx, ggml_tensor *a, int lp0, int rp0, int lp1, int rp1, int lp2, int rp2,
                          int lp3, int rp3) {
    const int64_t ne[4] = {a->ne[0] + lp0 + rp0, a->ne[1] + lp1 + rp1, a->ne[2] + lp2 + rp2,
                           a->ne[3] + lp3 + rp3};
    ggml_tensor *t = node(ctx, GGML_OP_PAD, a->type, ne, a);
    const int32_t p[8] = {lp0, rp0, lp1, rp1, lp2, rp2, lp3, rp3};
    memcpy(t->op_params, p, sizeof p);
    return t;
}
ggml_tensor *ggml_upscale(ggml_context *ctx, ggml_tensor *a, int sf, ggml_scale_mode mode) {
    GGML_ASSERT(mode == GGML_SCALE_MODE_NEAREST && sf >= 1);
    const int64_t ne[4] = {a->ne[0] * sf, a->ne[1] * sf, a->ne[2], a->ne[3]};
    ggml_tensor *t = node(ctx, GGML_OP_UPSCALE, a->type, ne, a);
    t->op_params[0] = sf;
    return t;
}

// ---------------------------------------------------------------------------
// arithmetic constructors
// ---------------------------------------------------------------------------
static ggml_tensor *binary(ggml_context *ctx, ggml_op op, ggml_tensor *a, ggml_tensor *b) {
    for (int i = 0; i < 4; i++) GGML_ASSERT(a->ne[i] % b->ne[i] == 0);
    return node(ctx, op, a->type, a->ne, a, b);
}
ggml_tensor *ggml_add(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b) { return binary(ctx, GGML_OP_ADD, a, b); }
ggml_tensor *ggml_mul(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b) { return binary(ctx, GGML_OP_MUL, a, b); }
ggml_tensor *ggml_div(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b) { return binary(ctx, GGML_OP_DIV, a, b); }
ggml_tensor *ggml_sqr(ggml_context *ctx, ggml_tensor *a) { return node(ctx, GGML_OP_SQR, a->type, a->ne, a); }
ggml_tensor *ggml_sqrt(ggml_context *ctx, ggml_tensor *a) { return node(ctx, GGML_OP_SQRT, a->type, a->ne, a); }
ggml_tensor *ggml_tanh(ggml_context *ctx, ggml_tensor *a) { return node(ctx, GGML_OP_TANH, a->type, a->ne, a); }
ggml_tensor *ggml_sigmoid(ggml_context *ctx, ggml_tensor *a) {
    return node(ctx, GGML_OP_SIGMOID, a->type, a->ne, a);
}
ggml_tensor *ggml_leaky_relu(ggml_context *ctx, ggml_tensor *a, float slope, bool) {
    ggml_tensor *t = node(ctx, GGML_OP_LEAKY_RELU, a->type, a->ne, a);
    memcpy(t->op_params, &slope, 4);
    return t;
}
ggml_tensor *ggml_scale_bias(ggml_context *ctx, ggml_tensor *a, float s, float b) {
    ggml_tensor *t = node(ctx, GGML_OP_SCALE_BIAS, a->type, a->ne, a);
    memcpy(t->op_params, &s, 4);
    memcpy(t->op_params + 1, &b, 4);
    return t;
}
ggml_tensor *ggml_norm(ggml_context *ctx, ggml_tensor *a, float eps) {
    ggml_tensor *t = node(ctx, GGML_OP_NORM, a->type, a->ne, a);
    memcpy(t->op_params, &eps, 4);
    return t;
}
ggml_tensor *ggml_mul_mat(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b) {
    GGML_ASSERT(a->ne[0] == b->ne[0]);
    GGML_ASSERT(b->ne[2] % a->ne[2] == 0 && b->ne[3] % a->ne[3] == 0);
    const int64_t ne[4] = {a->ne[1], b->ne[1], b->ne[2], b->ne[3]};
    return node(ctx, GGML_OP_MUL_MAT, GGML_TYPE_F32, ne, a, b);
}

// ---------------------------------------------------------------------------
// convolution constructors
// ---------------------------------------------------------------------------
ggml_tensor *ggml_im2col(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b, int s0, int s1, int p0, int p1, int d0,
                         int d1, bool is_2D, ggml_type dst_type) {
    GGML_ASSERT(is_2D);  // the reference's graphs use the 2-D form only
    GGML_ASSERT(a->ne[2] == b->ne[2]);
    const int64_t OH = ggml_calc_conv_output_size(b->ne[1], a->ne[1], s1, p1, d1);
    const int64_t OW = ggml_calc_conv_output_size(b->ne[0], a->ne[0], s0, p0, d0);
    const int64_t ne[4] = {a->ne[2] * a->ne[1] * a->ne[0], OW, OH, b->ne[3]};
    ggml_tensor *t = node(ctx, GGML_OP_IM2COL, dst_type, ne, a, b);
    const int32_t p[7] = {s0, s1, p0, p1, d0, d1, 1};
    memcpy(t->op_params, p, sizeof p);
    return t;
}
ggml_tensor *ggml_conv_2d_direct(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b, int s0, int s1, int p0, int p1,
                                 int d0, int d1) {
    GGML_ASSERT(a->ne[2] == b->ne[2]);
    const int64_t ne[4] = {ggml_calc_conv_output_size(b->ne[0], a->ne[0], s0, p0, d0),
                           ggml_calc_conv_output_size(b->ne[1], a->ne[1], s1, p1, d1), a->ne[3], b->ne[3]};
    ggml_tensor *t = node(ctx, GGML_OP_CONV_2D, GGML_TYPE_F32, ne, a, b);
    const int32_t p[6] = {s0, s1, p0, p1, d0, d1};
    memcpy(t->op_params, p, sizeof p);
    return t;
}
ggml_tensor *ggml_conv_2d_dw_direct(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b, int s0, int s1, int p0,
                                    int p1, int d0, int d1) {
    GGML_ASSERT(a->ne[2] == 1 && a->ne[3] == b->ne[2]);
    const int64_t ne[4] = {ggml_calc_conv_output_size(b->ne[0], a->ne[0], s0, p0, d0),
                           ggml_calc_conv_output_size(b->ne[1], a->ne[1], s1, p1, d1), b->ne[2], b->ne[3]};
    ggml_tensor *t = node(ctx, GGML_OP_CONV_2D_DW, b->type, ne, a, b);
    const int32_t p[6] = {s0, s1, p0, p1, d0, d1};
    memcpy(t->op_params, p, sizeof p);
    return t;
}
ggml_tensor *ggml_conv_transpose_2d_p0(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b, int stride) {
    GGML_ASSERT(a->ne[3] == b->ne[2]);
    const int64_t ne[4] = {(b->ne[0] - 1) * stride + a->ne[0], (b->ne[1] - 1) * stride + a->ne[1], a->ne[2],
                           b->ne[3]};
    ggml_tensor *t = node(ctx, GGML_OP_CONV_TRANSPOSE_2D, GGML_TYPE_F32, ne, a, b);
    t->op_params[0] = stride;
    return t;
}

// ---------------------------------------------------------------------------
// graphs
// ---------------------------------------------------------------------------
ggml_cgraph *ggml_new_graph_custom(ggml_context *ctx, size_t, bool) {
    ctx->graphs.push_back(std::make_unique<ggml_cgraph>());
    return ctx->graphs.back().get();
}
static void visit(ggml_cgraph *g, ggml_tensor *t) {
    if (!t || g->seen.count(t)) return;
    g->seen.insert(t);
    for (ggml_tensor *s : t->src) visit(g, s);
    if (t->op != GGML_OP_NONE) g->nodes.push_back(t);
}
void ggml_build_forward_expand(ggml_cgraph *gf, ggml_tensor *t) { visit(gf, t); }
int ggml_graph_n_nodes(ggml_cgraph *gf) { return (int) gf->nodes.size(); }
ggml_tensor *ggml_graph_node(ggml_cgraph *gf, int i) { return gf->nodes[(size_t) (i < 0 ? gf->nodes.size() + i : i)]; }

// ---------------------------------------------------------------------------
// host "backend" buffers
// ---------------------------------------------------------------------------
ggml_backend_buffer_t ggml_backend_alloc_ctx_tensors(ggml_context *ctx, ggml_backend_t) {
    auto *b = new ggml_backend_buffer();
    for (auto &t : ctx->tensors) {
        if (t->data || t->view_src) continue;
        t->data = calloc(1, ggml_nbytes(t.get()));
        t->owns_data = true;
        b->owned.push_back(t.get());
    }
    return b;
}
void ggml_backend_buffer_free(ggml_backend_buffer_t buf) {
    if (!buf) return;
    for (ggml_tensor *t : buf->owned) free_data(t);
    delete buf;
}
void ggml_backend_tensor_set(ggml_tensor *t, const void *data, size_t offset, size_t size) {
    GGML_ASSERT(t->data && offset + size <= ggml_nbytes(t));
    memcpy((char *) t->data + offset, data, size);
}
void ggml_backend_tensor_get(const ggml_tensor *t, void *data, size_t offset, size_t size) {
    GGML_ASSERT(t->data && offset + size <= ggml_nbytes(t));
    memcpy(data, (const char *) t->data + offset, size);
}

// ---------------------------------------------------------------------------
// evaluation
// ---------------------------------------------------------------------------
namespace {

inline const char *at(const ggml_tensor *t, int64_t i0, int64_t i1, int64_t i2, int64_t i3) {
    return (const char *) t->data + i0 * t->nb[0] + i1 * t->nb[1] + i2 * t->nb[2] + i3 * t->nb[3];
}
inline float ldf(const ggml_tensor *t, const char *p) {
    return t->type == GGML_TYPE_F16 ? ggml_fp16_to_fp32(*(const ggml_fp16_t *) p) : *(const float *) p;
}
inline void stf(const ggml_tensor *t, char *p, float v) {
    if (t->type == GGML_TYPE_F16)
        *(ggml_fp16_t *) p = ggml_fp32_to_fp16(v);
    else
        *(float *) p = v;
}

// a contiguous f32 copy of any tensor (optionally rounded through f16)
std::vector<float> to_f32(const ggml_tensor *t, bool round16 = false) {
    std::vector<float> v((size_t) ggml_nelements(t));
    const int64_t n0 = t->ne[0], n1 = t->ne[1], n2 = t->ne[2], n3 = t->ne[3];
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t i3 = 0; i3 < n3; i3++)
        for (int64_t i2 = 0; i2 < n2; i2++)
            for (int64_t i1 = 0; i1 < n1; i1++) {
                float *d = v.data() + ((i3 * n2 + i2) * n1 + i1) * n0;
                for (int64_t i0 = 0; i0 < n0; i0++) {
                    const float x = ldf(t, at(t, i0, i1, i2, i3));
                    d[i0] = round16 ? round_f16(x) : x;
                }
            }
    return v;
}

// elementwise over dst (contiguous) with a per-element function of the index
template <typename F>
void each(ggml_tensor *d, F &&f) {
    const int64_t n0 = d->ne[0], n1 = d->ne[1], n2 = d->ne[2], n3 = d->ne[3];
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t i3 = 0; i3 < n3; i3++)
        for (int64_t i2 = 0; i2 < n2; i2++)
            for (int64_t i1 = 0; i1 < n1; i1++)
                for (int64_t i0 = 0; i0 < n0; i0++)
                    stf(d, (char *) at(d, i0, i1, i2, i3), f(i0, i1, i2, i3));
}

float unary(ggml_op op, float x, const ggml_tensor *d) {
    switch (op) {
        case GGML_OP_SQR: return x * x;
        case GGML_OP_SQRT: return sqrtf(x);
        case GGML_OP_TANH: return tanhf(x);
        case GGML_OP_SIGMOID: return 1.0f / (1.0f + expf(-x));
        case GGML_OP_LEAKY_RELU: {
            float s;
            memcpy(&s, d->op_params, 4);
            return x > 0.0f ? x : s * x;
        }
        case GGML_OP_SCALE_BIAS: {
            float s, b;
            memcpy(&s, d->op_params, 4);
            memcpy(&b, d->op_params + 1, 4);
            return x * s + b;
        }
        default: throw std::runtime_error("unary op");
    }
}

// C[m][n] = sum_k A[m][k] * B[n][k], rows contiguous (K floats each)
void gemm_nt(const float *A, const float *B, float *C, int64_t M, int64_t N, int64_t K, int64_t ldc) {
    constexpr int TM = 4, TN = 4;
#pragma omp parallel for collapse(2) schedule(dynamic, 4)
    for (int64_t n0 = 0; n0 < N; n0 += TN)
        for (int64_t m0 = 0; m0 < M; m0 += TM) {
            const int mm = (int) std::min<int64_t>(TM, M - m0), nn = (int) std::min<int64_t>(TN, N - n0);
            float acc[TM][TN][8] = {};
            const float *a[TM], *b[TN];
            for (int i = 0; i < TM; i++) a[i] = A + (m0 + std::min(i, mm - 1)) * K;
            for (int j = 0; j < TN; j++) b[j] = B + (n0 + std::min(j, nn - 1)) * K;
            int64_t k = 0;
            for (; k + 8 <= K; k += 8)
                for (int i = 0; i < TM; i++)
                    for (int j = 0; j < TN; j++)
#pragma omp simd
                        for (int l = 0; l < 8; l++) acc[i][j][l] += a[i][k + l] * b[j][k + l];
            for (int i = 0; i < mm; i++)
                for (int j = 0; j < nn; j++) {
                    float s = 0.0f;
                    for (int l = 0; l < 8; l++) s += acc[i][j][l];
                    for (int64_t kk = k; kk < K; kk++) s += a[i][kk] * b[j][kk];
                    C[(n0 + j) * ldc + m0 + i] = s;
                }
        }
}

void eval_mul_mat(ggml_tensor *d) {
    const ggml_tensor *a = d->src[0], *b = d->src[1];
    const bool f16 = a->type == GGML_TYPE_F16;
    const std::vector<float> A = to_f32(a), B = to_f32(b, f16);
    const int64_t K = a->ne[0], M = a->ne[1], N = b->ne[1];
    const int64_t r2 = b->ne[2] / a->ne[2], r3 = b->ne[3] / a->ne[3];
    for (int64_t i3 = 0; i3 < b->ne[3]; i3++)
        for (int64_t i2 = 0; i2 < b->ne[2]; i2++) {
            const float *pa = A.data() + ((i3 / r3) * a->ne[2] + i2 / r2) * M * K;
            const float *pb = B.data() + (i3 * b->ne[2] + i2) * N * K;
            float *pc = (float *) d->data + (i3 * b->ne[2] + i2) * M * N;
            gemm_nt(pa, pb, pc, M, N, K, M);
        }
}

// direct conv: per (n, oc block, output row), accumulate input rows
void eval_conv2d(ggml_tensor *d) {
    const ggml_tensor *a = d->src[0], *b = d->src[1];
    const int32_t *p = d->op_params;
    const int s0 = p[0], s1 = p[1], p0 = p[2], p1 = p[3], d0 = p[4], d1 = p[5];
    const std::vector<float> K = to_f32(a), X = to_f32(b, a->type == GGML_TYPE_F16);
    const int64_t KW = a->ne[0], KH = a->ne[1], IC = a->ne[2], OC = a->ne[3];
    const int64_t IW = b->ne[0], IH = b->ne[1], NB = b->ne[3];
    const int64_t OW = d->ne[0], OH = d->ne[1];
    constexpr int OB = 4;
    float *out = (float *) d->data;
#pragma omp parallel for collapse(3) schedule(dynamic, 1)
    for (int64_t n = 0; n < NB; n++)
        for (int64_t oc0 = 0; oc0 < OC; oc0 += OB)
            for (int64_t oy = 0; oy < OH; oy++) {
                const int ob = (int) std::min<int64_t>(OB, OC - oc0);
                std::vector<float> acc((size_t) OB * OW, 0.0f);
                for (int64_t ic = 0; ic < IC; ic++)
                    for (int64_t kh = 0; kh < KH; kh++) {
                        const int64_t iy = oy * s1 + kh * d1 - p1;
                        if (iy < 0 || iy >= IH) continue;
                        const float *row = X.data() + ((n * IC + ic) * IH + iy) * IW;
                        for (int64_t kw = 0; kw < KW; kw++) {
                            // output columns whose input column is inside the map
                            const int64_t off = kw * d0 - p0;
                            int64_t lo = off >= 0 ? 0 : (-off + s0 - 1) / s0;
                            int64_t hi = (IW - 1 - off) >= 0 ? (IW - 1 - off) / s0 + 1 : 0;
                            hi = std::min(hi, OW);
                            for (int o = 0; o < ob; o++) {
                                const float w = K[(((oc0 + o) * IC + ic) * KH + kh) * KW + kw];
                                float *ac = acc.data() + (size_t) o * OW;
                                if (s0 == 1) {
                                    const float *r = row + off;
#pragma omp simd
                                    for (int64_t ox = lo; ox < hi; ox++) ac[ox] += w * r[ox];
                                } else {
                                    for (int64_t ox = lo; ox < hi; ox++) ac[ox] += w * row[ox * s0 + off];
                                }
                            }
                        }
                    }
                for (int o = 0; o < ob; o++)
                    memcpy(out + ((n * OC + oc0 + o) * OH + oy) * OW, acc.data() + (size_t) o * OW,
                           (size_t) OW * 4);
            }
}

void eval_conv2d_dw(ggml_tensor *d) {
    const ggml_tensor *a = d->src[0], *b = d->src[1];
    const int32_t *p = d->op_params;
    const int s0 = p[0], s1 = p[1], p0 = p[2], p1 = p[3], d0 = p[4], d1 = p[5];
    const std::vector<float> K = to_f32(a), X = to_f32(b);
    const int64_t KW = a->ne[0], KH = a->ne[1], C = b->ne[2];
    const int64_t IW = b->ne[0], IH = b->ne[1], NB = b->ne[3];
    const int64_t OW = d->ne[0], OH = d->ne[1];
    std::vector<float> out((size_t) ggml_nelements(d));
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t n = 0; n < NB; n++)
        for (int64_t c = 0; c < C; c++)
            for (int64_t oy = 0; oy < OH; oy++)
                for (int64_t ox = 0; ox < OW; ox++) {
                    float s = 0.0f;
                    for (int64_t kh = 0; kh < KH; kh++) {
                        const int64_t iy = oy * s1 + kh * d1 - p1;
                        if (iy < 0 || iy >= IH) continue;
                        for (int64_t kw = 0; kw < KW; kw++) {
                            const int64_t ix = ox * s0 + kw * d0 - p0;
                            if (ix < 0 || ix >= IW) continue;
                            s += K[(c * KH + kh) * KW + kw] * X[((n * C + c) * IH + iy) * IW + ix];
                        }
                    }
                    out[((n * C + c) * OH + oy) * OW + ox] = s;
                }
    each(d, [&](int64_t i0, int64_t i1, int64_t i2, int64_t i3) {
        return out[((i3 * C + i2) * OH + i1) * OW + i0];
    });
}

void eval_conv_transpose(ggml_tensor *d) {
    const ggml_tensor *a = d->src[0], *b = d->src[1];
    const int s = d->op_params[0];
    const std::vector<float> K = to_f32(a), X = to_f32(b, a->type == GGML_TYPE_F16);
    const int64_t KW = a->ne[0], KH = a->ne[1], OC = a->ne[2], IC = a->ne[3];
    const int64_t W = b->ne[0], H = b->ne[1], NB = b->ne[3];
    const int64_t OW = d->ne[0], OH = d->ne[1];
    float *out = (float *) d->data;
    memset(out, 0, ggml_nbytes(d));
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t n = 0; n < NB; n++)
        for (int64_t oc = 0; oc < OC; oc++)
            for (int64_t ic = 0; ic < IC; ic++)
                for (int64_t y = 0; y < H; y++)
                    for (int64_t x = 0; x < W; x++) {
                        const float v = X[((n * IC + ic) * H + y) * W + x];
                        for (int64_t ky = 0; ky < KH; ky++)
                            for (int64_t kx = 0; kx < KW; kx++)
                                out[((n * OC + oc) * OH + y * s + ky) * OW + x * s + kx] +=
                                    v * K[((ic * OC + oc) * KH + ky) * KW + kx];
                    }
}

void eval_im2col(ggml_tensor *d) {
    const ggml_tensor *a = d->src[0], *b = d->src[1];
    const int32_t *p = d->op_params;
    const int s0 = p[0], s1 = p[1], p0 = p[2], p1 = p[3], d0 = p[4], d1 = p[5];
    const bool cf = (p[6] & 2) != 0;
    const int64_t KW = a->ne[0], KH = a->ne[1];
    const int64_t IC = cf ? b->ne[0] : b->ne[2];
    const int64_t IW = cf ? b->ne[1] : b->ne[0], IH = cf ? b->ne[2] : b->ne[1], NB = b->ne[3];
    const int64_t OW = d->ne[1], OH = d->ne[2];
    const std::vector<float> X = to_f32(b);
    const int64_t R = IC * KH * KW;
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t n = 0; n < NB; n++)
        for (int64_t oy = 0; oy < OH; oy++)
            for (int64_t ox = 0; ox < OW; ox++) {
                char *row = (char *) at(d, 0, ox, oy, n);
                for (int64_t ic = 0; ic < IC; ic++)
                    for (int64_t kh = 0; kh < KH; kh++)
                        for (int64_t kw = 0; kw < KW; kw++) {
                            const int64_t iy = oy * s1 + kh * d1 - p1, ix = ox * s0 + kw * d0 - p0;
                            const bool in = iy >= 0 && iy < IH && ix >= 0 && ix < IW;
                            const int64_t r = cf ? ic + IC * (kw + KW * kh) : (ic * KH + kh) * KW + kw;
                            const float v = !in ? 0.0f
                                            : cf ? X[((n * IH + iy) * IW + ix) * IC + ic]
                                                 : X[((n * IC + ic) * IH + iy) * IW + ix];
                            (void) R;
                            stf(d, row + r * d->nb[0], v);
                        }
            }
}

void eval_norm(ggml_tensor *d) {
    const ggml_tensor *a = d->src[0];
    float eps;
    memcpy(&eps, d->op_params, 4);
    for (int64_t i3 = 0; i3 < a->ne[3]; i3++)
        for (int64_t i2 = 0; i2 < a->ne[2]; i2++)
            for (int64_t i1 = 0; i1 < a->ne[1]; i1++) {
                double s = 0.0, ss = 0.0;
                for (int64_t i0 = 0; i0 < a->ne[0]; i0++) s += ldf(a, at(a, i0, i1, i2, i3));
                const double mean = s / a->ne[0];
                for (int64_t i0 = 0; i0 < a->ne[0]; i0++) {
                    const double v = ldf(a, at(a, i0, i1, i2, i3)) - mean;
                    ss += v * v;
                }
                const double sc = 1.0 / std::sqrt(ss / a->ne[0] + eps);
                for (int64_t i0 = 0; i0 < a->ne[0]; i0++)
                    stf(d, (char *) at(d, i0, i1, i2, i3), (float) ((ldf(a, at(a, i0, i1, i2, i3)) - mean) * sc));
            }
}

void eval(ggml_tensor *d) {
    const ggml_tensor *a = d->src[0], *b = d->src[1];
    ggml_compute_params cp;
    switch (d->op) {
        case GGML_OP_DUP:
            each(d, [&](int64_t i0, int64_t i1, int64_t i2, int64_t i3) { return ldf(a, at(a, i0, i1, i2, i3)); });
            return;
        case GGML_OP_ADD:
        case GGML_OP_MUL:
        case GGML_OP_DIV: {
            const ggml_op op = d->op;
            each(d, [&](int64_t i0, int64_t i1, int64_t i2, int64_t i3) {
                const float x = ldf(a, at(a, i0, i1, i2, i3));
                const float y = ldf(b, at(b, i0 % b->ne[0], i1 % b->ne[1], i2 % b->ne[2], i3 % b->ne[3]));
                return op == GGML_OP_ADD ? x + y : op == GGML_OP_MUL ? x * y : x / y;
            });
            return;
        }
        case GGML_OP_SQR:
        case GGML_OP_SQRT:
        case GGML_OP_TANH:
        case GGML_OP_SIGMOID:
        case GGML_OP_LEAKY_RELU:
        case GGML_OP_SCALE_BIAS:
            each(d, [&](int64_t i0, int64_t i1, int64_t i2, int64_t i3) {
                return unary(d->op, ldf(a, at(a, i0, i1, i2, i3)), d);
            });
            return;
        case GGML_OP_CONCAT: {
            const int dim = d->op_params[0];
            each(d, [&](int64_t i0, int64_t i1, int64_t i2, int64_t i3) {
                int64_t i[4] = {i0, i1, i2, i3};
                if (i[dim] < a->ne[dim]) return ldf(a, at(a, i0, i1, i2, i3));
                i[dim] -= a->ne[dim];
                return ldf(b, at(b, i[0], i[1], i[2], i[3]));
            });
            return;
        }
        case GGML_OP_REPEAT:
            each(d, [&](int64_t i0, int64_t i1, int64_t i2, int64_t i3) {
                return ldf(a, at(a, i0 % a->ne[0], i1 % a->ne[1], i2 % a->ne[2], i3 % a->ne[3]));
            });
            return;
        case GGML_OP_PAD: {
            const int32_t *p = d->op_params;
            each(d, [&](int64_t i0, int64_t i1, int64_t i2, int64_t i3) {
                const int64_t j0 = i0 - p[0], j1 = i1 - p[2], j2 = i2 - p[4], j3 = i3 - p[6];
                if (j0 < 0 || j0 >= a->ne[0] || j1 < 0 || j1 >= a->ne[1] || j2 < 0 || j2 >= a->ne[2] || j3 < 0 ||
                    j3 >= a->ne[3])
                    return 0.0f;
                return ldf(a, at(a, j0, j1, j2, j3));
            });
            return;
        }
        case GGML_OP_UPSCALE: {
            const int sf = d->op_params[0];
            each(d, [&](int64_t i0, int64_t i1, int64_t i2, int64_t i3) {
                return ldf(a, at(a, i0 / sf, i1 / sf, i2, i3));
            });
            return;
        }
        case GGML_OP_MUL_MAT: eval_mul_mat(d); return;
        case GGML_OP_IM2COL: eval_im2col(d); return;
        case GGML_OP_CONV_2D: eval_conv2d(d); return;
        case GGML_OP_CONV_2D_DW: eval_conv2d_dw(d); return;
        case GGML_OP_CONV_TRANSPOSE_2D: eval_conv_transpose(d); return;
        case GGML_OP_NORM: eval_norm(d); return;
        case GGML_OP_BILINEAR_GATHER: ggml_compute_forward_bilinear_gather(&cp, d); return;
        case GGML_OP_BIAS_LRELU: ggml_compute_forward_bias_lrelu(&cp, d); return;
        case GGML_OP_SUBPIX_LRELU: ggml_compute_forward_subpix_lrelu(&cp, d); return;
        case GGML_OP_SUBPIX_LRELU_CL: ggml_compute_forward_subpix_lrelu_cl(&cp, d); return;
        case GGML_OP_UPFIRDN2X: ggml_compute_forward_upfirdn2x(&cp, d); return;
        case GGML_OP_CLSP_MUL: ggml_compute_forward_clsp_mul(&cp, d); return;
        case GGML_OP_CLSP_LERP: ggml_compute_forward_clsp_lerp(&cp, d); return;
        case GGML_OP_FLOW_GRID: ggml_compute_forward_flow_grid(&cp, d); return;
        default: throw std::runtime_error("stand-in: unhandled op " + std::to_string((int) d->op));
    }
}

bool is_alias(const ggml_tensor *t) { return t->view_src != nullptr; }
ggml_tensor *root_of(ggml_tensor *t) {
    while (t->view_src) t = t->view_src;
    return t;
}

}  // namespace

// Evaluate a graph: allocate each compute node when it runs, free it after
// its last consumer unless it is an output.
static void compute_graph(ggml_cgraph *g) {
    std::unordered_map<ggml_tensor *, int> refs;
    std::set<ggml_tensor *> keep;
    // an alias node uses no storage of its own: its consumers hold the root
    auto each_use = [](ggml_tensor *n, auto &&f) {
        for (ggml_tensor *s : n->src)
            if (s && !(is_alias(n) && s == n->view_src)) f(root_of(s));
    };
    for (ggml_tensor *n : g->nodes) {
        if (n->flags & GGML_TENSOR_FLAG_OUTPUT) keep.insert(root_of(n));
        each_use(n, [&](ggml_tensor *r) { refs[r]++; });
    }
    for (ggml_tensor *n : g->nodes)  // results of the previous compute
        if (!is_alias(n) && n->owns_data) free_data(n);
    for (ggml_tensor *n : g->nodes) {
        if (is_alias(n)) {
            n->data = (char *) n->view_src->data + n->view_offs;
        } else {
            n->data = calloc(1, ggml_nbytes(n));
            if (!n->data) throw std::runtime_error("stand-in: out of memory");
            n->owns_data = true;
            eval(n);
        }
        each_use(n, [&](ggml_tensor *r) {
            if (--refs[r] == 0 && r->op != GGML_OP_NONE && !keep.count(r) && r->owns_data) free_data(r);
        });
    }
}

// ---------------------------------------------------------------------------
// the reference runtime glue its decoder and encoder use
// ---------------------------------------------------------------------------
namespace tp {

bool backend_t::init(const char *, int n, std::string &) {
    n_threads = n;
    return true;
}
void backend_t::release() {}

void plan_t::begin(size_t max_nodes) {
    release();
    graph_size = max_nodes;
    ctx = ggml_init({0, nullptr, true});
    gf = ggml_new_graph_custom(ctx, max_nodes, false);
}

bool plan_t::commit(backend_t &, std::string &err) {
    try {
        for (ggml_tensor *t : outputs) ggml_build_forward_expand(gf, t);
        // graph inputs (leafs without storage) get their buffers now
        std::set<ggml_tensor *> seen;
        for (ggml_tensor *n : gf->nodes)
            for (ggml_tensor *s : n->src)
                if (s && s->op == GGML_OP_NONE && !s->data && !seen.count(s)) {
                    seen.insert(s);
                    s->data = calloc(1, ggml_nbytes(s));
                    s->owns_data = true;
                }
        // view nodes of storage that exists now
        for (ggml_tensor *n : gf->nodes)
            if (n->view_src && n->view_src->data) n->data = (char *) n->view_src->data + n->view_offs;
    } catch (const std::exception &e) {
        err = e.what();
        return false;
    }
    return true;
}

bool plan_t::compute(backend_t &, std::string &err) {
    try {
        compute_graph(gf);
    } catch (const std::exception &e) {
        err = e.what();
        return false;
    }
    return true;
}

void plan_t::release() {
    if (ctx) ggml_free(ctx);
    ctx = nullptr;
    gf = nullptr;
    galloc = nullptr;
    sched = nullptr;
    named.clear();
    outputs.clear();
}

bool read_file(const std::string &path, std::vector<uint8_t> &out, std::string &err) {
    std::ifstream f(path, std::ios::binary | std::ios::ate);
    if (!f) {
        err = "cannot open " + path;
        return false;
    }
    const std::streamsize n = f.tellg();
    f.seekg(0);
    out.resize((size_t) n);
    if (n && !f.read((char *) out.data(), n)) {
        err = "short read on " + path;
        return false;
    }
    return true;
}

ggml_tensor *linear(ggml_context *ctx, ggml_tensor *W, ggml_tensor *b, ggml_tensor *x) {
    ggml_tensor *y = ggml_mul_mat(ctx, W, x);
    return b ? ggml_add(ctx, y, b) : y;
}

ggml_tensor *layer_norm(ggml_context *ctx, ggml_tensor *x, ggml_tensor *w, ggml_tensor *b, float eps) {
    x = ggml_norm(ctx, x, eps);
    if (w) x = ggml_mul(ctx, x, w);
    if (b) x = ggml_add(ctx, x, b);
    return x;
}

// taps are copied out as contiguous f32 arrays keyed by name
bool tap_sink::harvest() {
    for (auto &e : pending) {
        std::vector<float> v = to_f32(e.t);
        wr->taps[e.name] = std::move(v);
    }
    pending.clear();
    return true;
}

}  // namespace tp
