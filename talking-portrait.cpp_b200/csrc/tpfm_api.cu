// Flow-matching sampler C ABI (include/tpfm.h): fmt_model::forward
// (src/fmt.cpp:64-211) and sample_chunk_ex (src/pipeline.cpp:15-91). The
// plain linears run on the library's tcgen05 GEMM (kernels_gemm_tc.cu;
// row-major Y[M][N] = X[M][K] W[N][K]^T): f16 operands in the f16 mode, the
// three-pass TF32 split in the f32 mode. The block linears add their bias
// in the GEMM epilogue (fc1 also applies GELU); the embedding, adaLN and
// output linears run without bias and the kernel consuming their output
// adds it. The adaLN modulations of all blocks and of the final layer depend
// only on the conditioning, so one GEMM per forward computes them together
// (their weights are contiguous in the arena). Norms, banded attention, gated
// residuals and the CFG/Euler update are the kernels of kernels_fmt.cu. A
// chunk's nine forwards run as one captured CUDA graph.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/tpfm.h"
#include "tpmd_internal.h"

namespace tpmd {
cudaError_t fmt_gemv(const float *W, const float *x, const float *b, int N, int K, bool silu_act, float *y,
                     cudaStream_t st);
cudaError_t fmt_cond_silu(bool f16, const float *clin, const float *bc, const float *te, int M, int H, void *sc,
                          cudaStream_t st);
// with x1: x = x1[m mod T] + bx + pos[m mod T] first (stored), then the norm
cudaError_t fmt_norm_mod(bool f16, float *x, int M, int H, float eps, const float *mod, const float *bmod,
                         int mod_stride, int shift_off, int scale_off, void *h, cudaStream_t st,
                         const float *x1 = nullptr, const float *bx = nullptr, const float *pos = nullptr,
                         int T = 0);
cudaError_t fmt_attn(bool f16, const float *qkv, int T, int H, int nh, int window, void *out, cudaStream_t st);
cudaError_t fmt_res_norm(bool f16, float *x, const float *o, const float *mod, const float *bmod,
                         int mod_stride, int gate_off, int M, int H, float eps, const float *mod2, const float *bmod2,
                         int shift_off, int scale_off, void *h, cudaStream_t st);
cudaError_t fmt_cfg_euler(const float *vout, const float *bv, int T, int P, int D, float a_cfg, float e_cfg,
                          float dt, float *x, float *x60, __half *x60h, cudaStream_t st);
cudaError_t fmt_add_bias(const float *a, const float *b, int M, int N, float *y, cudaStream_t st);
cudaError_t fmt_to_half(const float *a, int64_t n, __half *y, cudaStream_t st);
}  // namespace tpmd

using namespace tpmd;

namespace {
thread_local std::string g_create_err;

// torch linspace(0,1,nfe) in f32, as src/pipeline.cpp:13 computes it
float ode_t(int i, int nfe) { return (float) ((double) i / (double) (nfe - 1)); }
}  // namespace

struct tpfm_ctx {
    int device = 0;
    bool f16 = false;
    tpfm_config c{};
    int T = 0, M = 0, CD = 0, CDp = 0, FF = 0, H = 0;  // CDp: CD padded to 8 (GEMM row strides)
    int nmod = 0;  // adaLN columns of all blocks + the final layer
    std::string err;
    std::map<std::string, int64_t> spec;
    std::map<std::string, std::vector<float>> host;
    std::map<std::string, size_t> off32, off16;
    std::map<std::string, int> kdim, ldk;  // linear weights: K, and the row stride (K padded to 8)
    float *w32 = nullptr;
    __half *w16 = nullptr;
    bool wready = false;
    cudaStream_t stream = nullptr;
    void *act = nullptr;
    int *gerr = nullptr;  // the GEMMs' error flag
    float *x60 = nullptr, *cond = nullptr, *clin = nullptr, *te0 = nullptr, *te = nullptr, *x1 = nullptr,
          *x = nullptr, *mod = nullptr, *qkv = nullptr, *o = nullptr,
          *vout = nullptr, *v = nullptr, *xc = nullptr, *tf = nullptr,
          *te_all = nullptr;  // timestep embedding of every sampler step (prepare)
    void *sc = nullptr, *h = nullptr, *att = nullptr, *m1 = nullptr, *cond_in = nullptr, *x60_in = nullptr;
    cudaGraphExec_t graph = nullptr;

    bool fail(const std::string &m) {
        err = m;
        return false;
    }
    bool ck(cudaError_t e, const char *what) {
        if (e == cudaSuccess) return true;
        err = std::string(what) + ": " + cudaGetErrorString(e);
        cudaGetLastError();
        return false;
    }
    const float *F(const std::string &n) const { return w32 + off32.at(n); }
    const void *Wt(const std::string &n) const {
        return f16 ? (const void *) (w16 + off16.at(n)) : (const void *) F(n);
    }
    // Y[M][N] (f32, or f16 into Yh) = epi(X[M][K] (GEMM input type) W[N][K]^T)
    // with row strides ldx, ldw; epi adds bias and applies act (gemm_desc)
    bool gemm_w(const void *X, int Mr, int K, int ldx, const void *W, int ldw, int N, float *Y, const char *what,
                const float *bias = nullptr, int act = 0, __half *Yh = nullptr) {
        gemm_desc d;
        d.f32 = !f16;
        d.X = X;
        d.ldx = ldx;
        d.W = W;
        d.ldw = ldw;
        d.Y = Yh ? nullptr : Y;
        d.Yh = Yh;
        d.ldy = N;
        d.M = Mr;
        d.N = N;
        d.K = K;
        d.bias = bias;
        d.act = act;
        d.err = gerr;
        d.pdl = d.w_const = true;  // W: weights; the forward's kernels are programmatic dependents
        return ck(gemm_tc(d, stream), what);
    }
    bool gemm(const void *X, int Mr, int K, const std::string &wname, int N, float *Y, const float *bias = nullptr) {
        return gemm_w(X, Mr, K, K, Wt(wname), ldk.at(wname), N, Y, wname.c_str(), bias);
    }
    // after a synchronize: a GEMM whose pipeline wait expired
    bool gemm_status() {
        int flag = 0;
        if (!ck(cudaMemcpy(&flag, gerr, sizeof flag, cudaMemcpyDeviceToHost), "GEMM status")) return false;
        if (!flag) return true;
        cudaMemset(gerr, 0, sizeof(int));
        return fail("a GEMM pipeline wait timed out");
    }
    // the first adaLN weight: all depth + 1 of them are contiguous from here
    const void *adaln_w() const { return Wt("blocks.0.adaLN_modulation.1.weight"); }
    ~tpfm_ctx() {
        if (device >= 0) cudaSetDevice(device);
        if (graph) cudaGraphExecDestroy(graph);
        if (gerr) cudaFree(gerr);
        if (act) cudaFree(act);
        if (w32) cudaFree(w32);
        if (w16) cudaFree(w16);
        if (stream) cudaStreamDestroy(stream);
    }
};

namespace {

void build_spec(tpfm_ctx *c) {
    const int H = c->H;
    auto lin = [&](const std::string &n, int64_t out, int64_t in) {
        c->spec[n + ".weight"] = out * in;
        c->spec[n + ".bias"] = out;
        c->kdim[n + ".weight"] = (int) in;
        c->ldk[n + ".weight"] = (int) ((in + 7) & ~(int64_t) 7);
    };
    lin("t_embedder.mlp.0", H, c->c.t_freq_dim);
    lin("t_embedder.mlp.2", H, H);
    lin("c_embedder", H, c->CD);
    lin("x_embedder.proj", H, c->c.dim_w);
    c->spec["pos_embed"] = (int64_t) c->T * H;
    for (int i = 0; i < c->c.depth; i++) {
        const std::string b = "blocks." + std::to_string(i) + ".";
        lin(b + "adaLN_modulation.1", 6 * H, H);
        lin(b + "attn.qkv", 3 * H, H);
        lin(b + "attn.proj", H, H);
        lin(b + "mlp.fc1", c->FF, H);
        lin(b + "mlp.fc2", H, c->FF);
    }
    lin("decoder.adaLN_modulation.1", 2 * H, H);
    lin("decoder.linear", c->c.dim_w, H);
}

// the weights that go through the GEMM (kept f16 in f16 mode)
bool is_gemm_weight(const std::string &n) {
    const size_t k = n.size();
    return k > 7 && n.compare(k - 7, 7, ".weight") == 0 && n.rfind("t_embedder.", 0) != 0;
}

// the timestep MLP of tf row `s` into te (two GEMVs)
bool t_embed(tpfm_ctx *c, int s, float *te) {
    const int H = c->H;
    const float *tf = c->tf + (size_t) s * c->c.t_freq_dim;
    return c->ck(fmt_gemv(c->F("t_embedder.mlp.0.weight"), tf, c->F("t_embedder.mlp.0.bias"), H, c->c.t_freq_dim,
                          true, c->te0, c->stream),
                 "t embed") &&
           c->ck(fmt_gemv(c->F("t_embedder.mlp.2.weight"), c->te0, c->F("t_embedder.mlp.2.bias"), H, H, false, te,
                          c->stream),
                 "t embed");
}

// one forward on the device buffers: x60 (f32) and the chunk's clin are set;
// tf row `s`; output in vout (no bias). in_chunk: a sampler step, whose
// timestep embedding was computed at prepare and whose x60 f16 copy the
// chunk keeps current; otherwise both are formed here.
bool forward_device(tpfm_ctx *c, int s, bool in_chunk = false) {
    cudaStream_t st = c->stream;
    const int H = c->H, T = c->T, M = c->M, FF = c->FF;
    const bool h16 = c->f16;
    auto K = [&](cudaError_t e, const char *w) { return c->ck(e, w); };
    const float *te = in_chunk ? c->te_all + (size_t) s * H : c->te;
    if ((!in_chunk && !t_embed(c, s, c->te)) ||
        !K(fmt_cond_silu(h16, c->clin, c->F("c_embedder.bias"), te, M, H, c->sc, st), "cond silu"))
        return false;
    const void *x60_in = c->x60;
    if (h16) {
        if (!in_chunk &&
            !K(fmt_to_half(c->x60, (int64_t) T * c->c.dim_w, (__half *) c->x60_in, st), "x60 f16"))
            return false;
        x60_in = c->x60_in;
    }
    const int NM = c->nmod;
    if (!c->gemm(x60_in, T, c->c.dim_w, "x_embedder.proj.weight", H, c->x1) ||
        !c->gemm_w(c->sc, M, H, H, c->adaln_w(), H, NM, c->mod, "adaLN modulation"))
        return false;
    // each gated residual runs fused with the layer norm after it; the first
    // block's attention norm forms the embedded rows (x1 + bias + pos, three
    // branches) itself
    const float eps = c->c.ln_eps;
    if (!K(fmt_norm_mod(h16, c->x, M, H, eps, c->mod, c->F("blocks.0.adaLN_modulation.1.bias"), NM, 0, H, c->h, st,
                        c->x1, c->F("x_embedder.proj.bias"), c->F("pos_embed"), T),
           "embed + norm"))
        return false;
    for (int l = 0; l < c->c.depth; l++) {
        const std::string b = "blocks." + std::to_string(l) + ".";
        const float *bmod = c->F(b + "adaLN_modulation.1.bias");
        const float *md = c->mod + (size_t) l * 6 * H;  // this block's six modulation vectors
        // the norm after the MLP residual: the next block's attention norm, or the final layer's
        const bool last = l + 1 == c->c.depth;
        const float *md2 = c->mod + (size_t) (l + 1) * 6 * H;
        const float *bmod2 = last ? c->F("decoder.adaLN_modulation.1.bias")
                                  : c->F("blocks." + std::to_string(l + 1) + ".adaLN_modulation.1.bias");
        if (!c->gemm(c->h, M, H, b + "attn.qkv.weight", 3 * H, c->qkv, c->F(b + "attn.qkv.bias")) ||
            !K(fmt_attn(h16, c->qkv, T, H, c->c.n_heads, c->c.attn_window, c->att, st), "attention") ||
            !c->gemm(c->att, M, H, b + "attn.proj.weight", H, c->o, c->F(b + "attn.proj.bias")) ||
            !K(fmt_res_norm(h16, c->x, c->o, md, bmod, NM, 2 * H, M, H, eps, md, bmod,
                            3 * H, 4 * H, c->h, st),
               "residual + norm") ||
            // m1 = gelu_tanh(h fc1^T + bias), in the GEMM input type
            !c->gemm_w(c->h, M, H, H, c->Wt(b + "mlp.fc1.weight"), c->ldk.at(b + "mlp.fc1.weight"), FF,
                       h16 ? nullptr : (float *) c->m1, "mlp.fc1", c->F(b + "mlp.fc1.bias"), 2,
                       h16 ? (__half *) c->m1 : nullptr) ||
            !c->gemm(c->m1, M, FF, b + "mlp.fc2.weight", H, c->o, c->F(b + "mlp.fc2.bias")) ||
            !K(fmt_res_norm(h16, c->x, c->o, md, bmod, NM, 5 * H, M, H, eps, md2, bmod2, 0,
                            H, c->h, st),
               "residual + norm"))
            return false;
    }
    return c->gemm(c->h, M, H, "decoder.linear.weight", c->c.dim_w, c->vout);
}

// clin = cond . c_embedder^T (the conditioning rows, fixed for a chunk)
bool embed_cond(tpfm_ctx *c) {
    const void *in = c->cond;
    if (c->f16) {
        if (!c->ck(fmt_to_half(c->cond, (int64_t) c->M * c->CDp, (__half *) c->cond_in, c->stream), "cond f16"))
            return false;
        in = c->cond_in;
    }
    return c->gemm_w(in, c->M, c->CD, c->CDp, c->Wt("c_embedder.weight"), c->ldk.at("c_embedder.weight"), c->H,
                     c->clin, "c_embedder");
}

bool ready(tpfm_ctx *c) {
    if (!c->wready) return c->fail("weights not prepared (tpfm_prepare)");
    return c->ck(cudaSetDevice(c->device), "cudaSetDevice");
}

}  // namespace

extern "C" {

void tpfm_default_config(tpfm_config *cfg) {
    if (!cfg) return;
    *cfg = tpfm_config{1024, 8, 8, 512, 512, 7, 50, 10, 2, 256, 10, 4.0f, 1e-6f, 2.0f, 1.0f};
}

tpfm_ctx *tpfm_create(int device, int dtype, const tpfm_config *cfg) {
    int n = 0;
    if (!cfg || (dtype != TPMD_DTYPE_F32 && dtype != TPMD_DTYPE_F16)) {
        g_create_err = "tpfm_create: bad argument";
        return nullptr;
    }
    if (cfg->dim_h <= 0 || cfg->n_heads <= 0 || cfg->dim_h % cfg->n_heads || cfg->depth <= 0 || cfg->nfe < 2 ||
        cfg->chunk_frames <= 0 || cfg->prev_frames < 0 || cfg->attn_window < 0 || 2 * cfg->attn_window + 1 > 16 ||
        cfg->t_freq_dim < 2 || cfg->t_freq_dim % 2 || cfg->dim_w <= 0 || cfg->dim_a < 0 || cfg->dim_e < 0 ||
        cfg->mlp_ratio <= 0.0f || cfg->dim_h % 8 || cfg->dim_w % 8 || (int) (cfg->dim_h * cfg->mlp_ratio) % 8) {
        g_create_err = "tpfm_create: invalid config";
        return nullptr;
    }
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
        cudaGetLastError();
        g_create_err = "tpfm_create: no such CUDA device";
        return nullptr;
    }
    cudaDeviceProp pr{};
    if (cudaGetDeviceProperties(&pr, device) != cudaSuccess || pr.major != 10) {
        cudaGetLastError();
        g_create_err = "tpfm_create: needs an sm_100 (B200) GPU";
        return nullptr;
    }
    tpfm_ctx *c = new tpfm_ctx();
    c->device = device;
    c->f16 = dtype == TPMD_DTYPE_F16;
    c->c = *cfg;
    c->H = cfg->dim_h;
    c->T = cfg->chunk_frames + cfg->prev_frames;
    c->M = 3 * c->T;
    c->CD = cfg->dim_w + cfg->dim_a + cfg->dim_e;
    c->CDp = (c->CD + 7) & ~7;
    c->FF = (int) (cfg->dim_h * cfg->mlp_ratio);
    c->nmod = cfg->depth * 6 * cfg->dim_h + 2 * cfg->dim_h;
    build_spec(c);
    // activations
    const size_t H = c->H, T = c->T, M = c->M, D = cfg->dim_w, FF = c->FF, CD = c->CDp;
    const size_t es = c->f16 ? 2 : 4;
    size_t sizes[] = {T * D * 4, M * CD * 4, M * H * 4, H * 4, H * 4, T * H * 4, M * H * 4, M * (size_t) c->nmod * 4,
                      M * 3 * H * 4, M * H * 4, M * D * 4, M * D * 4,
                      (size_t) cfg->chunk_frames * D * 4, (size_t) (cfg->nfe) * cfg->t_freq_dim * 4,
                      (size_t) cfg->nfe * H * 4,
                      M * H * es, M * H * es, M * H * es, M * FF * es, M * CD * es, T * D * es};
    const int ns = sizeof(sizes) / sizeof(sizes[0]);
    size_t offs[32], total = 0;
    for (int i = 0; i < ns; i++) {
        offs[i] = total;
        total += (sizes[i] + 255) & ~(size_t) 255;
    }
    bool ok = c->ck(cudaSetDevice(device), "cudaSetDevice") &&
              c->ck(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking), "stream") &&
              c->ck(cudaMalloc(&c->act, total), "cudaMalloc(fmt activations)") &&
              c->ck(cudaMemset(c->act, 0, total), "cudaMemset(fmt activations)") &&
              c->ck(cudaMalloc(&c->gerr, sizeof(int)), "cudaMalloc(GEMM flag)") &&
              c->ck(cudaMemset(c->gerr, 0, sizeof(int)), "cudaMemset(GEMM flag)") &&
              c->ck(gemm_tc_prepare(), "GEMM set-up");
    if (!ok) {
        g_create_err = c->err;
        delete c;
        return nullptr;
    }
    char *b = (char *) c->act;
    int i = 0;
    float **fl[] = {&c->x60, &c->cond, &c->clin, &c->te0, &c->te, &c->x1, &c->x, &c->mod, &c->qkv, &c->o,
                    &c->vout, &c->v, &c->xc, &c->tf, &c->te_all};
    for (float **p : fl) *p = (float *) (b + offs[i++]);
    void **vp[] = {&c->sc, &c->h, &c->att, &c->m1, &c->cond_in, &c->x60_in};
    for (void **p : vp) *p = b + offs[i++];
    // the t-embedding frequencies of every Euler step (host, as the reference)
    const int half = cfg->t_freq_dim / 2;
    std::vector<float> tf((size_t) cfg->nfe * cfg->t_freq_dim);
    for (int s = 0; s < cfg->nfe; s++) {
        const float t = ode_t(s, cfg->nfe);
        for (int k = 0; k < half; k++) {
            const float fr = (float) exp(-log(10000.0) * (double) k / (double) half);
            tf[(size_t) s * cfg->t_freq_dim + k] = cosf(t * fr);
            tf[(size_t) s * cfg->t_freq_dim + half + k] = sinf(t * fr);
        }
    }
    if (!c->ck(cudaMemcpy(c->tf, tf.data(), tf.size() * 4, cudaMemcpyHostToDevice), "t freqs")) {
        g_create_err = c->err;
        delete c;
        return nullptr;
    }
    return c;
}

const char *tpfm_create_error(void) { return g_create_err.c_str(); }
void tpfm_destroy(tpfm_ctx *c) { delete c; }
const char *tpfm_last_error(const tpfm_ctx *c) { return c ? c->err.c_str() : "no context"; }

int tpfm_set_tensor(tpfm_ctx *c, const char *name, const float *data, int64_t n) {
    if (!c) return -1;
    if (!name || !data) return c->fail("tpfm_set_tensor: null argument"), -1;
    auto it = c->spec.find(name);
    if (it == c->spec.end()) return c->fail(std::string("tpfm_set_tensor: unknown tensor ") + name), -1;
    if (it->second != n)
        return c->fail(std::string("tpfm_set_tensor: size mismatch for ") + name + " (want " +
                       std::to_string(it->second) + ", got " + std::to_string(n) + ")"),
               -1;
    c->host[name].assign(data, data + n);
    c->wready = false;
    return 0;
}

}  // extern "C"

namespace {
struct kv_check {
    tpfm_ctx *c;
    std::string bad;
};
// float.fmt.* keys (src/fmt.cpp:10-26) against the handle's config
int check_kv(void *user, const char *key, int, double num, const char *) {
    kv_check *k = (kv_check *) user;
    const tpfm_config &g = k->c->c;
    const std::string s = key;
    if (s.rfind("float.fmt.", 0) != 0) return 0;
    const std::string n = s.substr(10);
    const std::map<std::string, double> want = {
        {"dim_h", g.dim_h}, {"depth", g.depth}, {"n_heads", g.n_heads}, {"dim_w", g.dim_w}, {"dim_a", g.dim_a},
        {"dim_e", g.dim_e}, {"chunk_frames", g.chunk_frames}, {"prev_frames", g.prev_frames},
        {"num_total_frames", g.chunk_frames + g.prev_frames}, {"attn_window", g.attn_window},
        {"t_freq_dim", g.t_freq_dim}, {"nfe", g.nfe}, {"a_cfg_scale", g.a_cfg}, {"e_cfg_scale", g.e_cfg},
        {"ln_eps", g.ln_eps}, {"mlp_ratio", g.mlp_ratio}};
    auto it = want.find(n);
    if (it == want.end()) return 0;
    if (std::fabs(num - it->second) > 1e-6 * std::max(1.0, std::fabs(it->second))) {
        k->bad = s + " = " + std::to_string(num) + " differs from the handle's " + std::to_string(it->second);
        return 1;
    }
    return 0;
}
int take_fmt_tensor(void *user, const char *name, const int64_t *, const float *data, int64_t n) {
    tpfm_ctx *c = (tpfm_ctx *) user;
    if (!c->spec.count(name)) return 0;  // not part of the model
    return tpfm_set_tensor(c, name, data, n);
}
}  // namespace

extern "C" {

int tpfm_load_gguf(tpfm_ctx *c, const char *path) {
    if (!c) return -1;
    char e[1024] = {0};
    kv_check k{c, ""};
    if (tpmd_gguf_read_kv(path, "float-fmt", check_kv, &k, e, sizeof e) != 0) {
        c->fail(k.bad.empty() ? std::string(e) : std::string(path) + ": " + k.bad);
        return -1;
    }
    if (tpmd_gguf_read(path, "float-fmt", 0, take_fmt_tensor, c, e, sizeof e) != 0) {
        if (std::string(e).find("rejected by the consumer") == std::string::npos) c->fail(e);
        return -1;
    }
    return 0;
}

int tpfm_prepare(tpfm_ctx *c) {
    if (!c) return -1;
    for (auto &kv : c->spec)
        if (!c->host.count(kv.first)) return c->fail("tpfm_prepare: missing tensor " + kv.first), -1;
    size_t n32 = 0, n16 = 0;
    c->off32.clear();
    c->off16.clear();
    // the adaLN weights of every block and of the final layer first, back to
    // back in that order: one GEMM computes all the modulations
    std::vector<std::string> order;
    for (int l = 0; l < c->c.depth; l++) order.push_back("blocks." + std::to_string(l) + ".adaLN_modulation.1.weight");
    order.push_back("decoder.adaLN_modulation.1.weight");
    for (auto &kv : c->spec)
        if (std::find(order.begin(), order.end(), kv.first) == order.end()) order.push_back(kv.first);
    const size_t n_adaln = (size_t) c->c.depth + 1;
    // GEMM weights are stored with rows padded to ldk (16-byte row strides)
    auto padded = [&](const std::string &n) { return is_gemm_weight(n) && c->ldk.at(n) != c->kdim.at(n); };
    auto stored = [&](const std::string &n) {
        return padded(n) ? (size_t) (c->spec.at(n) / c->kdim.at(n)) * c->ldk.at(n) : (size_t) c->spec.at(n);
    };
    for (size_t i = 0; i < order.size(); i++) {
        const std::string &n = order[i];
        const size_t sz = stored(n);
        c->off32[n] = n32;
        n32 += sz;
        if (c->f16 && is_gemm_weight(n)) {
            c->off16[n] = n16;
            n16 += sz;
        }
        if (i + 1 >= n_adaln) {  // 256-byte aligned starts after the adaLN group
            n32 = (n32 + 63) & ~(size_t) 63;
            n16 = (n16 + 127) & ~(size_t) 127;
        }
    }
    std::vector<float> img(n32, 0.0f);
    for (auto &kv : c->spec) {
        const std::string &n = kv.first;
        if (!padded(n)) {
            memcpy(img.data() + c->off32[n], c->host[n].data(), kv.second * 4);
            continue;
        }
        const int64_t K = c->kdim.at(n), ld = c->ldk.at(n);
        for (int64_t r = 0; r < kv.second / K; r++)
            memcpy(img.data() + c->off32[n] + r * ld, c->host[n].data() + r * K, K * 4);
    }
    if (!c->ck(cudaSetDevice(c->device), "cudaSetDevice")) return -1;
    if (c->w32) cudaFree(c->w32);
    if (c->w16) cudaFree(c->w16);
    c->w32 = nullptr;
    c->w16 = nullptr;
    if (c->graph) {
        cudaGraphExecDestroy(c->graph);
        c->graph = nullptr;
    }
    if (!c->ck(cudaMalloc(&c->w32, n32 * 4), "cudaMalloc(fmt weights)") ||
        !c->ck(cudaMemcpy(c->w32, img.data(), n32 * 4, cudaMemcpyHostToDevice), "upload fmt weights"))
        return -1;
    if (c->f16) {
        if (!c->ck(cudaMalloc(&c->w16, n16 * 2), "cudaMalloc(fmt f16 weights)")) return -1;
        for (auto &kv : c->off16)
            if (!c->ck(fmt_to_half(c->w32 + c->off32[kv.first], (int64_t) stored(kv.first), c->w16 + kv.second,
                                   c->stream),
                       "f16 weights"))
                return -1;
        if (!c->ck(cudaStreamSynchronize(c->stream), "f16 weights")) return -1;
    }
    // the sampler's timestep embeddings depend only on the weights
    for (int s = 0; s + 1 < c->c.nfe; s++)
        if (!t_embed(c, s, c->te_all + (size_t) s * c->H)) return -1;
    if (!c->ck(cudaStreamSynchronize(c->stream), "t embeddings")) return -1;
    c->wready = true;
    return 0;
}

static int tpfm_forward_enqueue(tpfm_ctx *c, const float *x60, const float *cond, float t, float *v) {
    if (!c) return -1;
    if (!x60 || !cond || !v) return c->fail("tpfm_forward: null argument"), -1;
    if (!ready(c)) return -1;
    // the t-embedding row for this t
    const int half = c->c.t_freq_dim / 2;
    std::vector<float> tf((size_t) c->c.t_freq_dim);
    for (int k = 0; k < half; k++) {
        const float fr = (float) exp(-log(10000.0) * (double) k / (double) half);
        tf[(size_t) k] = cosf(t * fr);
        tf[(size_t) half + k] = sinf(t * fr);
    }
    // a spare row past the sampler's steps holds it
    float *row = c->tf + (size_t) (c->c.nfe - 1) * c->c.t_freq_dim;
    cudaStream_t st = c->stream;
    const size_t D = c->c.dim_w;
    if (!c->ck(cudaMemcpyAsync(row, tf.data(), tf.size() * 4, cudaMemcpyHostToDevice, st), "t freq") ||
        !c->ck(cudaMemcpyAsync(c->x60, x60, (size_t) c->T * D * 4, cudaMemcpyHostToDevice, st), "x60") ||
        !c->ck(cudaMemcpy2DAsync(c->cond, (size_t) c->CDp * 4, cond, (size_t) c->CD * 4, (size_t) c->CD * 4,
                                 (size_t) c->M, cudaMemcpyHostToDevice, st),
               "cond") ||
        !embed_cond(c) || !forward_device(c, c->c.nfe - 1) ||
        !c->ck(fmt_add_bias(c->vout, c->F("decoder.linear.bias"), c->M, (int) D, c->v, st), "bias") ||
        !c->ck(cudaMemcpyAsync(v, c->v, (size_t) c->M * D * 4, cudaMemcpyDeviceToHost, st), "v D2H") ||
        !c->ck(cudaStreamSynchronize(st), "forward") || !c->gemm_status())
        return -1;
    return 0;
}

// On a failure after work was enqueued, the stream is drained before the
// call returns, so no copy reads or writes the caller's buffers after it.
int tpfm_forward(tpfm_ctx *c, const float *x60, const float *cond, float t, float *v) {
    const int rc = tpfm_forward_enqueue(c, x60, cond, t, v);
    if (rc != 0 && c && c->stream) cudaStreamSynchronize(c->stream);
    return rc;
}

static int tpfm_sample_chunk_enqueue(tpfm_ctx *c, const float *wr, const float *prev_wa, const float *cond_audio,
                                     const float *prev_x, const float *x0, int emotion, float *motion) {
    if (!c) return -1;
    if (!wr || !cond_audio || !x0 || !motion || (c->c.prev_frames > 0 && (!prev_wa || !prev_x)))
        return c->fail("tpfm_sample_chunk: null argument"), -1;
    if (!ready(c)) return -1;
    // rows of CDp floats (the GEMM's padded row stride), padding zero
    const int T = c->T, P = c->c.prev_frames, CF = c->c.chunk_frames, D = c->c.dim_w, CD = c->CDp;
    // condition rows [wr | wa | we] per branch: uncond nulls the current
    // frames' wa and we, audio-only nulls we; prev_wa rows stay in all
    std::vector<float> cond((size_t) 3 * T * CD, 0.0f);
    for (int b = 0; b < 3; b++)
        for (int f = 0; f < T; f++) {
            float *row = cond.data() + ((size_t) b * T + f) * CD;
            memcpy(row, wr, (size_t) D * 4);
            const float *wa = f < P ? prev_wa + (size_t) f * D : cond_audio + (size_t) (f - P) * D;
            if (!(b == 0 && f >= P)) memcpy(row + D, wa, (size_t) D * 4);
            if (b == 1 && emotion >= 0 && emotion < c->c.dim_e) row[D + c->c.dim_a + emotion] = 1.0f;
        }
    cudaStream_t st = c->stream;
    if ((P > 0 && !c->ck(cudaMemcpyAsync(c->x60, prev_x, (size_t) P * D * 4, cudaMemcpyHostToDevice, st), "prev_x")) ||
        !c->ck(cudaMemcpyAsync(c->x60 + (size_t) P * D, x0, (size_t) CF * D * 4, cudaMemcpyHostToDevice, st), "x0") ||
        !c->ck(cudaMemcpyAsync(c->xc, x0, (size_t) CF * D * 4, cudaMemcpyHostToDevice, st), "x0") ||
        !c->ck(cudaMemcpyAsync(c->cond, cond.data(), cond.size() * 4, cudaMemcpyHostToDevice, st), "cond"))
        return -1;
    if (!c->graph) {
        // capture the chunk's device work once; buffers are fixed per handle
        cudaGraph_t g = nullptr;
        if (!c->ck(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal), "begin capture")) return -1;
        // the f16 copy of x60 is made once here; each Euler step refreshes its rows
        bool ok = embed_cond(c) &&
                  (!c->f16 || c->ck(fmt_to_half(c->x60, (int64_t) T * D, (__half *) c->x60_in, st), "x60 f16"));
        for (int s = 0; ok && s < c->c.nfe - 1; s++) {
            const float dt = ode_t(s + 1, c->c.nfe) - ode_t(s, c->c.nfe);
            ok = forward_device(c, s, true) &&
                 c->ck(fmt_cfg_euler(c->vout, c->F("decoder.linear.bias"), T, P, D, c->c.a_cfg, c->c.e_cfg, dt, c->xc,
                                     c->x60, c->f16 ? (__half *) c->x60_in : nullptr, st),
                       "cfg euler");
        }
        const cudaError_t e = cudaStreamEndCapture(st, &g);
        if (!ok) {
            if (g) cudaGraphDestroy(g);
            return -1;
        }
        if (!c->ck(e, "end capture")) return -1;
        const cudaError_t ie = cudaGraphInstantiate(&c->graph, g, 0);
        cudaGraphDestroy(g);
        if (!c->ck(ie, "instantiate")) return -1;
    }
    if (!c->ck(cudaGraphLaunch(c->graph, st), "graph launch") ||
        !c->ck(cudaMemcpyAsync(motion, c->xc, (size_t) CF * D * 4, cudaMemcpyDeviceToHost, st), "motion D2H") ||
        !c->ck(cudaStreamSynchronize(st), "sample chunk") || !c->gemm_status())
        return -1;
    return 0;
}

// On a failure after work was enqueued, the stream is drained before the
// call returns, so no copy reads or writes the caller's buffers after it.
int tpfm_sample_chunk(tpfm_ctx *c, const float *wr, const float *prev_wa, const float *cond_audio,
                      const float *prev_x, const float *x0, int emotion, float *motion) {
    const int rc = tpfm_sample_chunk_enqueue(c, wr, prev_wa, cond_audio, prev_x, x0, emotion, motion);
    if (rc != 0 && c && c->stream) cudaStreamSynchronize(c->stream);
    return rc;
}

}  // extern "C"
