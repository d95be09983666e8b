// tpmd C ABI: handle lifecycle, weight derivation, device arenas and the
// batched decode loop. Replaces the reference's motion_dec
// (src/motion_dec.h:10-49, src/motion_dec.cpp:31-226 and 659-1220) and the
// ggml plan/backend glue it runs on (src/backend.cpp:68-189).
//
// Design (B200-first, not a graph interpreter):
//  * all decoder weights live in one device arena laid out at create time
//    (prepare fills it; multi-GPU ranks receive it by broadcast), the feats in
//    a second arena, activations in a workspace sized for max_batch frames:
//    zero allocations after set-up, as the reference's plan pattern requires;
//  * one decode of nb frames is a fixed sequence of 25 kernels (style, den,
//    conv1 input, conv1, then per level: up-conv, conv2, tail) captured once
//    per (nb, input, output) into a CUDA graph and replayed;
//  * the host entry point splits n frames into sub-batches and overlaps each
//    sub-batch's device-to-host frame copy (second stream) with the next
//    sub-batch's compute, double-buffering the device staging frames.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <list>
#include <mutex>
#include <map>
#include <new>
#include <string>
#include <thread>
#include <vector>

#include "../../include/tpmd.h"
#include "tpmd_internal.h"

using namespace tpmd;

namespace {

thread_local std::string g_create_err;

size_t align256(size_t v) { return (v + 255) & ~(size_t) 255; }
// pixels over all levels (8x8 .. 512x512): one projected-feats float4 each
size_t proj_count() {
    size_t n = 0;
    for (int j = 0; j < N_LEVELS; j++) n += (size_t) (8 << j) * (8 << j);
    return n;
}

struct conv_layout {
    std::string name;  // weight tensor name
    std::string base;  // module base ("dec.conv1", "dec.convs.N")
    int IC = 0, OC = 0;
    bool up = false;
    size_t wg = 0, saug = 0, abias = 0;  // byte offsets in the weight arena
    int s_off = 0;                       // input style offset in a frame's s_all row
    int d_off = 0;                       // inv_den offset in a frame's row
};

struct stage_layout {
    size_t fW = 0, fb = 0, fup = 0, rW = 0, rlb = 0, rb = 0, rup = 0, lin = 0;
    int fs_off = 0;  // ToFlow style offset
};

// the per-decode scratch a chunk runs in: the handle's workspace, or the
// static array of tpmd_decode_noalloc
struct ws_view {
    float *s_all, *inv_den;
    void *actA, *actB, *actC;
    float *sf[2], *sk[2];
    int *err;
    bool timed;          // record CUDA events around each launch (live profiling)
    long long stall_ns;  // test hook armed for this chunk's first tcgen05 conv (0: none)
};

struct graph_entry {
    int64_t nb;
    const void *styles;
    void *out;
    int last;           // last level enqueued
    const void *split;  // split_in::trunk of a tail-levels chunk, else null
    cudaGraphExec_t exec;
};

// The inputs of a chunk that runs only the last two levels (r256, r512) of
// frames whose earlier levels ran in an earlier chunk: that chunk's r128
// trunk and skip planes of the first frame of this one. The r256 trunk then
// goes to the conv2 buffer (unused by the fused levels), so the earlier
// chunk's trunk and skips stay intact for the chunks that follow.
struct split_in {
    const void *trunk;
    const float *sf, *sk;
};
constexpr int SPLIT_LEVEL = N_LEVELS - 2;  // the first level of a tail-levels chunk

}  // namespace

struct tpmd_ctx {
    int device = 0, dtype = 0, max_batch = 0;
    bool f16 = false;
    bool use_tc = false;     // tcgen05 convs (f16 mode)
    bool use_graph = true;
    cudaStream_t stream = nullptr, copy_stream = nullptr, cap_stream = nullptr;
    cudaEvent_t ev_done[2] = {nullptr, nullptr}, ev_copied[2] = {nullptr, nullptr};
    // the end of the handle's last asynchronous decode (tpmd_decode_device),
    // on the caller's stream: the handle's later calls wait for it, so calls
    // on one handle use its workspace in call order on the GPU
    cudaEvent_t ev_order = nullptr;
    std::string err;

    std::map<std::string, int64_t> spec;
    std::map<std::string, std::vector<float>> host;

    conv_layout conv[N_CONVS];
    stage_layout stage[N_LEVELS];
    size_t off_wmod = 0, off_bmod = 0, off_input = 0;
    size_t feat_off[N_LEVELS] = {0};
    int S_TOT = 0, D_TOT = 0;
    den_table dtab{};

    void *warena = nullptr, *farena = nullptr;
    size_t wbytes = 0, fbytes = 0;
    bool wready = false, fready = false;
    // each level's feats projected by its ToRGB conv.0 weights ([r*r] float4
    // per level); lives after the feats arena (not broadcast: every rank
    // derives its own)
    float4 *proj = nullptr;
    size_t proj_off[N_LEVELS] = {0};  // in float4
    bool pready = false;

    // workspace
    void *ws = nullptr;
    size_t ws_bytes = 0;
    float *styles_d[2] = {nullptr, nullptr};
    float *s_all = nullptr, *inv_den = nullptr;
    void *actA = nullptr, *actB = nullptr, *actC = nullptr;
    float *sf[2] = {nullptr, nullptr}, *sk[2] = {nullptr, nullptr};
    float *frames_d[2] = {nullptr, nullptr};  // device staging for host decode
    uint8_t *rgb_d[2] = {nullptr, nullptr};   // RGB24 staging for tpmd_decode_rgb24
    int *err_flag = nullptr;                   // set by kernels whose bounded waits expired

    std::list<graph_entry> graphs;  // most recently used first
    long long stall_ns = 0;          // tpmd_debug_expire_wait: armed for the next decode

    // live profiling: (kernel name, start event, stop event) per launch
    bool profiling = false;
    struct prof_rec {
        std::string name;
        cudaEvent_t a, b;
    };
    std::vector<prof_rec> prof;

    size_t esz() const { return f16 ? 2 : 4; }
    char *W(size_t off) const { return (char *) warena + off; }
    const float *Wf(size_t off) const { return (const float *) ((char *) warena + off); }

    bool fail(const std::string &m) {
        err = m;
        return false;
    }
    bool ck(cudaError_t e, const char *what) {
        if (e == cudaSuccess) return true;
        err = std::string(what) + ": " + cudaGetErrorString(e);
        return false;
    }
    ~tpmd_ctx();
};

namespace {

std::map<std::string, int64_t> tensor_spec() {
    std::map<std::string, int64_t> m;
    char nm[64];
    m["dec.input.input"] = 512 * 16;
    m["dec.conv1.conv.weight"] = (int64_t) 512 * 512 * 9;
    m["dec.conv1.conv.modulation.weight"] = 512 * 512;
    m["dec.conv1.conv.modulation.bias"] = 512;
    m["dec.conv1.activate.bias"] = 512;
    for (int i = 0; i < 14; i++) {
        const int j = i / 2;
        const bool up = (i % 2) == 0;
        const int IC = up ? ST_IC[j] : ST_OC[j], OC = ST_OC[j];
        snprintf(nm, sizeof nm, "dec.convs.%d.conv.weight", i);
        m[nm] = (int64_t) OC * IC * 9;
        snprintf(nm, sizeof nm, "dec.convs.%d.conv.modulation.weight", i);
        m[nm] = (int64_t) IC * 512;
        snprintf(nm, sizeof nm, "dec.convs.%d.conv.modulation.bias", i);
        m[nm] = IC;
        snprintf(nm, sizeof nm, "dec.convs.%d.activate.bias", i);
        m[nm] = OC;
        if (up) {
            snprintf(nm, sizeof nm, "dec.convs.%d.conv.blur.kernel", i);
            m[nm] = 16;
        }
    }
    for (int j = 0; j < N_LEVELS; j++) {
        const int OC = ST_OC[j];
        snprintf(nm, sizeof nm, "dec.to_flows.%d.conv.weight", j);
        m[nm] = 3 * OC;
        snprintf(nm, sizeof nm, "dec.to_flows.%d.conv.modulation.weight", j);
        m[nm] = (int64_t) OC * 512;
        snprintf(nm, sizeof nm, "dec.to_flows.%d.conv.modulation.bias", j);
        m[nm] = OC;
        snprintf(nm, sizeof nm, "dec.to_flows.%d.bias", j);
        m[nm] = 3;
        snprintf(nm, sizeof nm, "dec.to_flows.%d.upsample.kernel", j);
        m[nm] = 16;
        snprintf(nm, sizeof nm, "dec.to_rgbs.%d.conv.0.weight", j);
        m[nm] = 3 * OC;
        snprintf(nm, sizeof nm, "dec.to_rgbs.%d.conv.1.bias", j);
        m[nm] = 3;
        snprintf(nm, sizeof nm, "dec.to_rgbs.%d.bias", j);
        m[nm] = 3;
        snprintf(nm, sizeof nm, "dec.to_rgbs.%d.upsample.kernel", j);
        m[nm] = 16;
    }
    return m;
}

// Arena layout. Style rows (s_all, one row of S_TOT floats per frame) are
// ordered conv1, convs.0..13, to_flows.0..6 (each its input-channel count);
// inv_den rows are conv1, convs.0..13 (each OC).
void build_layout(tpmd_ctx *c) {
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off = align256(off + bytes);
        return o;
    };
    int s = 0, d = 0;
    for (int k = 0; k < N_CONVS; k++) {
        conv_layout &L = c->conv[k];
        if (k == 0) {
            L.name = "dec.conv1.conv.weight";
            L.base = "dec.conv1";
            L.IC = L.OC = 512;
            L.up = false;
        } else {
            const int i = k - 1, j = i / 2;
            L.up = (i % 2) == 0;
            L.IC = L.up ? ST_IC[j] : ST_OC[j];
            L.OC = ST_OC[j];
            L.base = "dec.convs." + std::to_string(i);
            L.name = L.base + ".conv.weight";
        }
        const size_t N = (size_t) (L.up ? 4 : 1) * L.OC, K = (size_t) 9 * L.IC;
        L.wg = take(N * K * c->esz());
        L.saug = take((size_t) L.OC * (L.IC + 1) * 4);
        L.abias = take((size_t) L.OC * 4);
        L.s_off = s;
        s += L.IC;
        L.d_off = d;
        d += L.OC;
    }
    for (int j = 0; j < N_LEVELS; j++) {
        stage_layout &S = c->stage[j];
        const int OC = ST_OC[j], r = 8 << j;
        S.fW = take((size_t) 3 * OC * 4);
        S.fb = take(3 * 4);
        S.fup = take(16 * 4);
        S.rW = take((size_t) 3 * OC * 4);
        S.rlb = take(3 * 4);
        S.rb = take(3 * 4);
        S.rup = take(16 * 4);
        S.lin = take((size_t) r * 4);
        S.fs_off = s;
        s += OC;
    }
    c->S_TOT = s;
    c->D_TOT = d;
    c->off_wmod = take((size_t) s * STYLE_DIM * 4);
    c->off_bmod = take((size_t) s * 4);
    c->off_input = take((size_t) 16 * 512 * 4);
    c->wbytes = off;

    size_t foff = 0;
    for (int j = 0; j < N_LEVELS; j++) {
        const int r = 8 << j;
        c->feat_off[j] = foff;
        foff = align256(foff + (size_t) r * r * ST_OC[j] * c->esz());
    }
    c->fbytes = foff;

    den_table &t = c->dtab;
    t.n = N_CONVS;
    int row = 0;
    for (int k = 0; k < N_CONVS; k++) {
        t.row0[k] = row;
        row += c->conv[k].OC;
        t.ic[k] = c->conv[k].IC;
        t.saug_off[k] = (int64_t) (c->conv[k].saug / 4);
        t.s_off[k] = c->conv[k].s_off;
        t.d_off[k] = c->conv[k].d_off;
    }
    t.row0[N_CONVS] = row;
}

// per-frame activation elements of the three ping-pong buffers
void act_sizes(size_t &a, size_t &b, size_t &cc) {
    a = b = cc = (size_t) 16 * 512;  // conv1 input / output
    for (int j = 0; j < N_LEVELS; j++) {
        const size_t r = (size_t) 8 << j;
        const size_t lvl = r * r * ST_OC[j];
        cc = std::max(cc, lvl);                 // up-conv output
        a = std::max(a, lvl);                   // conv2 output
        if (j < N_LEVELS - 1) b = std::max(b, lvl);  // trunk
    }
}

bool alloc_workspace(tpmd_ctx *c) {
    const size_t B = (size_t) c->max_batch;
    size_t a, b, cc;
    act_sizes(a, b, cc);
    const size_t skip = (size_t) 3 * 256 * 256;  // largest stored skip level
    const size_t frame = (size_t) 3 * IMG * IMG;
    size_t off = 0;
    std::vector<size_t> offs;
    auto take = [&](size_t bytes) {
        offs.push_back(off);
        off = align256(off + bytes);
    };
    take(B * STYLE_DIM * 4);  // styles 0
    take(B * STYLE_DIM * 4);  // styles 1
    take(B * c->S_TOT * 4);
    take(B * c->D_TOT * 4);
    take(B * a * c->esz());
    take(B * b * c->esz());
    take(B * cc * c->esz());
    take(B * skip * 4);
    take(B * skip * 4);
    take(B * skip * 4);
    take(B * skip * 4);
    take(B * frame * 4);
    take(B * frame * 4);
    take(B * frame);  // RGB24 staging 0
    take(B * frame);  // RGB24 staging 1
    take(256);
    if (!c->ck(cudaMalloc(&c->ws, off), "cudaMalloc(workspace)")) return false;
    c->ws_bytes = off;
    char *p = (char *) c->ws;
    int i = 0;
    c->styles_d[0] = (float *) (p + offs[i++]);
    c->styles_d[1] = (float *) (p + offs[i++]);
    c->s_all = (float *) (p + offs[i++]);
    c->inv_den = (float *) (p + offs[i++]);
    c->actA = p + offs[i++];
    c->actB = p + offs[i++];
    c->actC = p + offs[i++];
    c->sf[0] = (float *) (p + offs[i++]);
    c->sf[1] = (float *) (p + offs[i++]);
    c->sk[0] = (float *) (p + offs[i++]);
    c->sk[1] = (float *) (p + offs[i++]);
    c->frames_d[0] = (float *) (p + offs[i++]);
    c->frames_d[1] = (float *) (p + offs[i++]);
    c->rgb_d[0] = (uint8_t *) (p + offs[i++]);
    c->rgb_d[1] = (uint8_t *) (p + offs[i++]);
    c->err_flag = (int *) (p + offs[i++]);
    return c->ck(cudaMemset(c->err_flag, 0, 256), "cudaMemset");
}

void to_half(const float *src, size_t n, __half *dst) {
    for (size_t i = 0; i < n; i++) dst[i] = __float2half_rn(src[i]);
}

// Derived weights on the host in double, as the reference's prepare does
// (src/motion_dec.cpp:101-224), written straight into the arena image.
void derive_conv(tpmd_ctx *c, const conv_layout &L, std::vector<char> &img) {
    const std::vector<float> &W = c->host.at(L.name);  // [OC][IC][3][3]
    const int IC = L.IC, OC = L.OC;
    const size_t K = (size_t) 9 * IC;
    // S_aug [OC][IC+1]: 0.5*sum W^2, 0.5e-8 (src/motion_dec.cpp:108-120)
    float *sa = (float *) (img.data() + L.saug);
    for (int o = 0; o < OC; o++) {
        for (int i = 0; i < IC; i++) {
            double s = 0;
            const float *pw = W.data() + ((size_t) o * IC + i) * 9;
            for (int k = 0; k < 9; k++) s += (double) pw[k] * pw[k];
            sa[(size_t) o * (IC + 1) + i] = (float) (s * 0.5);
        }
        sa[(size_t) o * (IC + 1) + IC] = 0.5e-8f;
    }
    // activate bias (already x sqrt2 by the load-time fold)
    memcpy(img.data() + L.abias, c->host.at(L.base + ".activate.bias").data(), (size_t) OC * 4);
    // GEMM matrix [N][K], k = (kh*3 + kw)*IC + ic
    const size_t N = (size_t) (L.up ? 4 : 1) * OC;
    std::vector<float> g(N * K);
    if (!L.up) {
        for (int o = 0; o < OC; o++)
            for (int i = 0; i < IC; i++)
                for (int t = 0; t < 9; t++) g[(size_t) o * K + (size_t) t * IC + i] = W[((size_t) o * IC + i) * 9 + t];
    } else {
        // conv_transpose(3x3, s2) then Blur(4x4, pad 1) per output parity class
        // (by, bx) = a 3x3 pad-1 conv of the input with
        // T[ty][tx] = sum_{cy,cx} V[cy][cx] * K[1+2ty-by-cy][1+2tx-bx-cx],
        // V the spatially flipped weight (src/motion_dec.cpp:144-191)
        const std::vector<float> &BK = c->host.at(L.base + ".conv.blur.kernel");
        std::vector<std::thread> th;
        const int nth = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
        for (int tix = 0; tix < nth; tix++) {
            th.emplace_back([&, tix] {
                for (int o = tix; o < OC; o += nth)
                    for (int i = 0; i < IC; i++) {
                        const float *pw = W.data() + ((size_t) o * IC + i) * 9;
                        for (int cls = 0; cls < 4; cls++) {
                            const int by = cls >> 1, bx = cls & 1;
                            float *dst = g.data() + (size_t) (cls * OC + o) * K;
                            for (int ty = 0; ty < 3; ty++)
                                for (int tx = 0; tx < 3; tx++) {
                                    double acc = 0;
                                    for (int cy = 0; cy < 3; cy++) {
                                        const int ay = 1 + 2 * ty - by - cy;
                                        if (ay < 0 || ay > 3) continue;
                                        for (int cx = 0; cx < 3; cx++) {
                                            const int ax = 1 + 2 * tx - bx - cx;
                                            if (ax < 0 || ax > 3) continue;
                                            acc += (double) pw[(2 - cy) * 3 + (2 - cx)] *
                                                   (double) BK[(size_t) ay * 4 + ax];
                                        }
                                    }
                                    dst[(size_t) (ty * 3 + tx) * IC + i] = (float) acc;
                                }
                        }
                    }
            });
        }
        for (auto &t : th) t.join();
    }
    if (c->f16)
        to_half(g.data(), g.size(), (__half *) (img.data() + L.wg));
    else
        memcpy(img.data() + L.wg, g.data(), g.size() * 4);
}

bool run_chunk(tpmd_ctx *c, const float *styles, int64_t nb, float *out, cudaStream_t st,
               int last_level = N_LEVELS - 1, const split_in *in = nullptr, int64_t row0 = 0);

}  // namespace

tpmd_ctx::~tpmd_ctx() {
    if (device >= 0) cudaSetDevice(device);
    for (auto &g : graphs) cudaGraphExecDestroy(g.exec);
    graphs.clear();
    for (int i = 0; i < 2; i++) {
        if (ev_done[i]) cudaEventDestroy(ev_done[i]);
        if (ev_copied[i]) cudaEventDestroy(ev_copied[i]);
    }
    if (ev_order) cudaEventDestroy(ev_order);
    for (auto &r : prof) {
        cudaEventDestroy(r.a);
        cudaEventDestroy(r.b);
    }
    if (ws) cudaFree(ws);
    if (warena) cudaFree(warena);
    if (farena) cudaFree(farena);
    if (stream) cudaStreamDestroy(stream);
    if (copy_stream) cudaStreamDestroy(copy_stream);
    if (cap_stream) cudaStreamDestroy(cap_stream);
}

extern "C" {

}  // extern "C"

// error text for entry points implemented in other files
__attribute__((visibility("hidden"))) int tpmd_ctx_fail(tpmd_ctx *c, const char *msg) {
    if (c) c->fail(msg);
    return -1;
}

extern "C" {

int tpmd_abi_version(void) { return TPMD_ABI_VERSION; }

const char *tpmd_create_error(void) { return g_create_err.c_str(); }

tpmd_ctx *tpmd_create(int device, int dtype, int max_batch) {
    g_create_err.clear();
    if (dtype != TPMD_DTYPE_F32 && dtype != TPMD_DTYPE_F16) {
        g_create_err = "dtype must be TPMD_DTYPE_F32 or TPMD_DTYPE_F16";
        return nullptr;
    }
    if (max_batch < 1 || max_batch > 256) {
        g_create_err = "max_batch must be in [1, 256]";
        return nullptr;
    }
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
        g_create_err = "no such CUDA device";
        cudaGetLastError();
        return nullptr;
    }
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major != 10) {
        g_create_err = "tpmd requires an sm_100 (B200-class) GPU";
        return nullptr;
    }
    tpmd_ctx *c = new (std::nothrow) tpmd_ctx();
    if (!c) {
        g_create_err = "out of host memory";
        return nullptr;
    }
    c->device = device;
    c->dtype = dtype;
    c->f16 = dtype == TPMD_DTYPE_F16;
    c->max_batch = max_batch;
    // f16 convs run on tcgen05; TPMD_CONV=simt selects the FFMA kernels
    // instead (an A/B knob, like the reference's TP_MDEC_* switches)
    const char *cv = getenv("TPMD_CONV");
    c->use_tc = c->f16 && !(cv && strcmp(cv, "simt") == 0);
    c->use_graph = getenv("TPMD_NO_GRAPH") == nullptr;
    c->spec = tensor_spec();
    build_layout(c);
    bool ok = c->ck(cudaSetDevice(device), "cudaSetDevice") &&
              c->ck(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking), "stream") &&
              c->ck(cudaStreamCreateWithFlags(&c->copy_stream, cudaStreamNonBlocking), "stream") &&
              c->ck(cudaStreamCreateWithFlags(&c->cap_stream, cudaStreamNonBlocking), "stream") &&
              c->ck(cudaMalloc(&c->warena, c->wbytes), "cudaMalloc(weights)") &&
              c->ck(cudaMalloc(&c->farena, c->fbytes + proj_count() * sizeof(float4)),
                    "cudaMalloc(feats)") &&
              alloc_workspace(c);
    if (ok) {
        c->proj = (float4 *) ((char *) c->farena + c->fbytes);
        size_t o = 0;
        for (int j = 0; j < N_LEVELS; j++) {
            c->proj_off[j] = o;
            o += (size_t) (8 << j) * (8 << j);
        }
    }
    for (int i = 0; ok && i < 2; i++)
        ok = c->ck(cudaEventCreateWithFlags(&c->ev_done[i], cudaEventDisableTiming), "event") &&
             c->ck(cudaEventCreateWithFlags(&c->ev_copied[i], cudaEventDisableTiming), "event");
    ok = ok && c->ck(cudaEventCreateWithFlags(&c->ev_order, cudaEventDisableTiming), "event");
    if (!ok) {
        g_create_err = c->err;
        delete c;
        return nullptr;
    }
    return c;
}

void tpmd_destroy(tpmd_ctx *c) { delete c; }

const char *tpmd_last_error(const tpmd_ctx *c) { return c ? c->err.c_str() : "no context"; }

double tpmd_scale_for(const char *cname, const int64_t *ne) {
    // motion_ae_scale, src/motion_enc.cpp:14-45
    if (!cname || !ne) return 1.0;
    const std::string name = cname;
    const double SQRT2 = 1.4142135623730951;
    auto ends = [&](const char *s) {
        const size_t n = strlen(s);
        return name.size() >= n && name.compare(name.size() - n, n, s) == 0;
    };
    auto starts = [&](const char *s) { return name.rfind(s, 0) == 0; };
    if (name == "enc.net_app.convs.0.1.bias" || ends(".conv1.1.bias") || ends(".activate.bias") ||
        (starts("dec.to_rgbs.") && ends(".conv.1.bias")))
        return SQRT2;
    if (!ends(".weight")) return 1.0;
    if (starts("dec.direction") || ends("noise.weight")) return 1.0;
    if (ends("modulation.weight") || starts("enc.fc.")) return 1.0 / sqrt((double) ne[0]);
    const double conv = 1.0 / sqrt((double) (ne[0] * ne[1] * ne[2]));
    if (name == "enc.net_app.convs.0.0.weight" || ends(".conv1.0.weight")) return conv * SQRT2;
    if (ends(".conv2.1.weight")) return conv;
    if (ends(".skip.1.weight")) return conv / SQRT2;
    if (name == "enc.net_app.convs.8.weight") return conv;
    if (starts("dec.to_rgbs.") && ends(".conv.0.weight")) return conv * SQRT2;
    if (ends(".conv.weight")) return conv;
    return 1.0;
}

int tpmd_set_tensor(tpmd_ctx *c, const char *name, const float *data, int64_t n) {
    if (!c) return -1;
    if (!name || !data) return c->fail("tpmd_set_tensor: null argument"), -1;
    auto it = c->spec.find(name);
    if (it == c->spec.end()) return c->fail(std::string("unknown tensor ") + name), -1;
    if (it->second != n)
        return c->fail(std::string(name) + ": expected " + std::to_string(it->second) +
                       " elements, got " + std::to_string(n)),
               -1;
    c->host[name].assign(data, data + n);
    return 0;
}

}  // extern "C"
namespace {
// Recomputed whenever the weights or the feats change (both must be set).
bool make_proj(tpmd_ctx *c) {
    c->pready = false;
    if (!c->wready || !c->fready) return true;
    if (!c->ck(cudaSetDevice(c->device), "cudaSetDevice")) return false;
    for (int j = 0; j < N_LEVELS; j++) {
        const int r = 8 << j;
        if (!c->ck(launch_project_feats(c->f16, (const char *) c->farena + c->feat_off[j],
                                        (int64_t) r * r, ST_OC[j], c->Wf(c->stage[j].rW),
                                        c->proj + c->proj_off[j], c->stream),
                   "project feats"))
            return false;
    }
    if (!c->ck(cudaStreamSynchronize(c->stream), "project feats")) return false;
    c->pready = true;
    return true;
}
}  // namespace
extern "C" {

int tpmd_prepare(tpmd_ctx *c) {
    if (!c) return -1;
    for (auto &kv : c->spec)
        if (!c->host.count(kv.first)) return c->fail("host copy missing for " + kv.first), -1;
    std::vector<char> img(c->wbytes, 0);
    for (int k = 0; k < N_CONVS; k++) derive_conv(c, c->conv[k], img);
    char nm[64];
    for (int j = 0; j < N_LEVELS; j++) {
        const stage_layout &S = c->stage[j];
        const int OC = ST_OC[j], r = 8 << j;
        auto put = [&](size_t off, const char *fmt, size_t n) {
            snprintf(nm, sizeof nm, fmt, j);
            memcpy(img.data() + off, c->host.at(nm).data(), n * 4);
        };
        put(S.fW, "dec.to_flows.%d.conv.weight", (size_t) 3 * OC);
        put(S.fb, "dec.to_flows.%d.bias", 3);
        put(S.fup, "dec.to_flows.%d.upsample.kernel", 16);
        put(S.rW, "dec.to_rgbs.%d.conv.0.weight", (size_t) 3 * OC);
        put(S.rlb, "dec.to_rgbs.%d.conv.1.bias", 3);
        put(S.rb, "dec.to_rgbs.%d.bias", 3);
        put(S.rup, "dec.to_rgbs.%d.upsample.kernel", 16);
        float *lin = (float *) (img.data() + S.lin);
        for (int i = 0; i < r; i++) lin[i] = (float) (-1.0 + 2.0 * i / (r - 1));
    }
    // modulation rows: conv1, convs.0..13, to_flows.0..6
    {
        float *wm = (float *) (img.data() + c->off_wmod);
        float *bm = (float *) (img.data() + c->off_bmod);
        size_t row = 0;
        auto put_mod = [&](const std::string &base, int ch) {
            memcpy(wm + row * STYLE_DIM, c->host.at(base + ".modulation.weight").data(),
                   (size_t) ch * STYLE_DIM * 4);
            memcpy(bm + row, c->host.at(base + ".modulation.bias").data(), (size_t) ch * 4);
            row += ch;
        };
        for (int k = 0; k < N_CONVS; k++) put_mod(c->conv[k].base + ".conv", c->conv[k].IC);
        for (int j = 0; j < N_LEVELS; j++)
            put_mod("dec.to_flows." + std::to_string(j) + ".conv", ST_OC[j]);
    }
    // constant input [512][4][4] (torch) -> pixel-major [16][512]
    {
        const std::vector<float> &in = c->host.at("dec.input.input");
        float *d = (float *) (img.data() + c->off_input);
        for (int ch = 0; ch < 512; ch++)
            for (int p = 0; p < 16; p++) d[p * 512 + ch] = in[(size_t) ch * 16 + p];
    }
    if (!c->ck(cudaSetDevice(c->device), "cudaSetDevice") ||
        !c->ck(cudaMemcpy(c->warena, img.data(), c->wbytes, cudaMemcpyHostToDevice),
               "upload weights"))
        return -1;
    c->wready = true;
    return make_proj(c) ? 0 : -1;
}

int tpmd_set_feats(tpmd_ctx *c, const float *const feats[TPMD_N_LEVELS]) {
    if (!c) return -1;
    if (!feats) return c->fail("tpmd_set_feats: null feats"), -1;
    std::vector<char> img(c->fbytes, 0);
    for (int j = 0; j < N_LEVELS; j++) {
        if (!feats[j]) return c->fail("tpmd_set_feats: null level"), -1;
        const size_t n = (size_t) (8 << j) * (8 << j) * ST_OC[j];
        if (c->f16)
            to_half(feats[j], n, (__half *) (img.data() + c->feat_off[j]));
        else
            memcpy(img.data() + c->feat_off[j], feats[j], n * 4);
    }
    if (!c->ck(cudaSetDevice(c->device), "cudaSetDevice") ||
        !c->ck(cudaMemcpy(c->farena, img.data(), c->fbytes, cudaMemcpyHostToDevice),
               "upload feats"))
        return -1;
    c->fready = true;
    return make_proj(c) ? 0 : -1;
}

int tpmd_set_feats_device(tpmd_ctx *c, const float *const feats_dev[TPMD_N_LEVELS], void *stream) {
    if (!c) return -1;
    if (!feats_dev) return c->fail("tpmd_set_feats_device: null feats"), -1;
    for (int j = 0; j < N_LEVELS; j++)
        if (!feats_dev[j]) return c->fail("tpmd_set_feats_device: null level"), -1;
    cudaStream_t st = (cudaStream_t) stream;
    if (!c->ck(cudaSetDevice(c->device), "cudaSetDevice")) return -1;
    for (int j = 0; j < N_LEVELS; j++) {
        const int64_t n = (int64_t) (8 << j) * (8 << j) * ST_OC[j];
        if (!c->ck(launch_convert_feats(feats_dev[j], n, c->f16, (char *) c->farena + c->feat_off[j], st),
                   "convert feats"))
            return -1;
    }
    if (!c->ck(cudaStreamSynchronize(st), "convert feats")) return -1;
    c->fready = true;
    return make_proj(c) ? 0 : -1;
}

int tpmd_batch(const tpmd_ctx *c) { return c ? c->max_batch : -1; }

int tpmd_arena(tpmd_ctx *c, int which, void **dev_ptr, size_t *bytes) {
    if (!c) return -1;
    if (!dev_ptr || !bytes || (which != 0 && which != 1)) return c->fail("tpmd_arena: bad argument"), -1;
    *dev_ptr = which == 0 ? c->warena : c->farena;
    *bytes = which == 0 ? c->wbytes : c->fbytes;
    return 0;
}

int tpmd_arena_adopt(tpmd_ctx *c, int which) {
    if (!c) return -1;
    if (which == 0)
        c->wready = true;
    else if (which == 1)
        c->fready = true;
    else
        return c->fail("tpmd_arena_adopt: bad argument"), -1;
    return make_proj(c) ? 0 : -1;
}

}  // extern "C"
namespace {
bool fused_level(const tpmd_ctx *c, int j);
}
extern "C" {

static int64_t tpmd_kernel_launches_impl(const tpmd_ctx *c, int64_t n) {
    if (!c || n <= 0) return 0;
    const int64_t chunks = (n + c->max_batch - 1) / c->max_batch;
    int per = 4 + 3 * N_LEVELS;
    for (int j = 0; j < N_LEVELS; j++) per -= fused_level(c, j) ? 1 : 0;
    return chunks * per;
}

}  // extern "C"

namespace {

// Enqueue the decode of nb frames: styles (device, [nb][512]) -> out (device,
// [nb][3][512][512]).
ws_view ctx_ws(const tpmd_ctx *c) {
    return ws_view{c->s_all, c->inv_den, c->actA, c->actB, c->actC,
                   {c->sf[0], c->sf[1]}, {c->sk[0], c->sk[1]}, c->err_flag,
                   c->profiling, 0};
}

// one kernel launch, bracketed by CUDA events while profiling
template <typename F>
bool launch(tpmd_ctx *c, bool timed, const std::string &name, cudaStream_t st, F &&fn) {
    cudaEvent_t a = nullptr, b = nullptr;
    if (timed) {
        if (!c->ck(cudaEventCreate(&a), "event") || !c->ck(cudaEventCreate(&b), "event") ||
            !c->ck(cudaEventRecord(a, st), "record"))
            return false;
    }
    if (!c->ck(fn(), name.c_str())) return false;
    if (timed) {
        if (!c->ck(cudaEventRecord(b, st), "record")) return false;
        c->prof.push_back({name, a, b});
    }
    return true;
}

// levels whose conv2 runs with the level tail fused into its epilogue
bool fused_level(const tpmd_ctx *c, int j) {
    return c->use_tc && conv_tail_tc_supported(ST_OC[j], ST_OC[j], 8 << j);
}

bool enqueue_chunk(tpmd_ctx *c, const ws_view &w, const float *styles, int64_t nb, float *out,
                   cudaStream_t st, int last_level = N_LEVELS - 1, bool keep_conv2 = false,
                   const split_in *in = nullptr) {
    const bool h = c->f16;
    const int B = (int) nb;
    // a tail-levels chunk: styles, denominators and levels up to r128 came from
    // an earlier chunk (w.s_all / w.inv_den point at this chunk's first frame)
    const int first = in ? SPLIT_LEVEL : 0;
    if (in && (keep_conv2 || last_level != N_LEVELS - 1 || !fused_level(c, SPLIT_LEVEL) ||
               !fused_level(c, N_LEVELS - 1)))
        return c->fail("tail-levels chunk: needs the fused tcgen05 levels"), false;
    if (!in && !launch(c, w.timed, "style", st, [&] {
            return launch_style(c->Wf(c->off_wmod), c->Wf(c->off_bmod), c->S_TOT, styles, B,
                                w.s_all, st);
        }))
        return false;
    if (!in && !launch(c, w.timed, "den", st, [&] {
            return launch_den((const float *) c->warena, c->dtab, w.s_all, c->S_TOT, B,
                              w.inv_den, c->D_TOT, st);
        }))
        return false;
    if (!in && !launch(c, w.timed, "conv1_input", st, [&] {
            return launch_conv1_input(h, c->Wf(c->off_input), w.s_all + c->conv[0].s_off,
                                      c->S_TOT, B, w.actA, st);
        }))
        return false;
    auto conv_p = [&](int k, const void *x, void *y, int Hh, const float *snext) {
        const conv_layout &L = c->conv[k];
        conv_params p{};
        p.x = x;
        p.w = c->W(L.wg);
        p.y = y;
        p.B = B;
        p.H = p.W = Hh;
        p.IC = L.IC;
        p.OC = L.OC;
        p.inv_den = w.inv_den + L.d_off;
        p.den_stride = c->D_TOT;
        p.bias = c->Wf(L.abias);
        p.snext = snext;
        p.snext_stride = c->S_TOT;
        p.err = w.err;
        p.stall_ns = k == 0 && c->use_tc ? w.stall_ns : 0;
        return p;
    };
    auto conv = [&](int k, const void *x, void *y, int Hh, const float *snext) {
        const conv_layout &L = c->conv[k];
        const conv_params p = conv_p(k, x, y, Hh, snext);
        std::string name = k == 0 ? "conv1" : (L.up ? "upconv_r" : "conv2_r") +
                                                   std::to_string(L.up ? 2 * Hh : Hh);
        return launch(c, w.timed, name, st, [&] {
            return c->use_tc ? launch_conv_tc(L.up, p, st) : launch_conv_simt(h, L.up, p, st);
        });
    };
    // conv1: 4x4 map, output x style of convs.0 -> trunk buffer
    if (!in && !conv(0, w.actA, w.actB, 4, w.s_all + c->conv[1].s_off)) return false;
    // trunk ping-pong: the tail writes its trunk where the up-conv read it
    // from (a tail-levels chunk: into the conv2 buffer)
    void *trunk = in ? w.actA : w.actB;
    for (int j = first; j <= last_level; j++) {
        const int r = 8 << j;
        const conv_layout &Lu = c->conv[1 + 2 * j], &Ld = c->conv[2 + 2 * j];
        const bool split_first = in && j == first;
        // up-conv: trunk (x its style) -> c1 (x conv2's style)
        if (!conv(1 + 2 * j, split_first ? in->trunk : trunk, w.actC, r / 2, w.s_all + Ld.s_off)) return false;
        (void) Lu;
        const bool fused = fused_level(c, j);
        // conv2: c1 -> out (unscaled, read by the tail)
        if (!fused && !conv(2 + 2 * j, w.actC, w.actA, r, nullptr)) return false;
        const stage_layout &S = c->stage[j];
        tail_params t{};
        t.out = w.actA;
        t.feat = (const char *) c->farena + c->feat_off[j];
        t.B = B;
        t.r = r;
        t.OC = ST_OC[j];
        t.fW = c->Wf(S.fW);
        t.fs = w.s_all + S.fs_off;
        t.s_stride = c->S_TOT;
        t.fb = c->Wf(S.fb);
        t.fup = c->Wf(S.fup);
        t.skipf_prev = split_first ? in->sf : j == 0 ? nullptr : w.sf[(j - 1) & 1];
        t.skipf_out = j == N_LEVELS - 1 ? nullptr : w.sf[j & 1];
        t.rW = c->Wf(S.rW);
        t.rlb = c->Wf(S.rlb);
        t.rb = c->Wf(S.rb);
        t.rup = c->Wf(S.rup);
        t.skip_prev = split_first ? in->sk : j == 0 ? nullptr : w.sk[(j - 1) & 1];
        t.skip_out = j == N_LEVELS - 1 ? out : w.sk[j & 1];
        t.lin = c->Wf(S.lin);
        t.trunk = j == N_LEVELS - 1 ? nullptr : trunk;
        t.snext = j == N_LEVELS - 1 ? nullptr : w.s_all + c->conv[3 + 2 * j].s_off;
        t.proj = c->proj + c->proj_off[j];
        if (fused) {
            const conv_params p = conv_p(2 + 2 * j, w.actC, keep_conv2 ? w.actA : nullptr, r, nullptr);
            if (!launch(c, w.timed, "conv2tail_r" + std::to_string(r), st,
                        [&] { return launch_conv_tail_tc(p, t, st); }))
                return false;
        } else if (!launch(c, w.timed, "tail_r" + std::to_string(r), st, [&] { return launch_tail(h, t, st); })) {
            return false;
        }
    }
    return true;
}

// One chunk: the whole decode of nb frames, or (last_level < the last) its
// levels up to last_level, or (in != null) the tail levels of the frames
// whose per-frame styles and denominators start at row row0 of the
// workspace. Launched from a cached CUDA graph where possible.
bool run_chunk(tpmd_ctx *c, const float *styles, int64_t nb, float *out, cudaStream_t st,
               int last_level, const split_in *in, int64_t row0) {
    nvtx_range range(in ? "tpmd chunk: r256-r512 part" : last_level < N_LEVELS - 1 ? "tpmd chunk: levels to r128"
                                                                                  : "tpmd chunk: all levels");
    ws_view w0 = ctx_ws(c);
    w0.s_all += row0 * c->S_TOT;
    w0.inv_den += row0 * c->D_TOT;
    if (c->stall_ns && !in) {  // the armed test hook runs once, outside any cached graph
        ws_view w = w0;
        w.stall_ns = c->stall_ns;
        c->stall_ns = 0;
        return enqueue_chunk(c, w, styles, nb, out, st, last_level);
    }
    if (!c->use_graph || c->profiling) return enqueue_chunk(c, w0, styles, nb, out, st, last_level, false, in);
    const void *split = in ? in->trunk : nullptr;
    for (auto it = c->graphs.begin(); it != c->graphs.end(); ++it) {
        if (it->nb == nb && it->styles == styles && it->out == out && it->last == last_level &&
            it->split == split) {
            c->graphs.splice(c->graphs.begin(), c->graphs, it);
            return c->ck(cudaGraphLaunch(c->graphs.front().exec, st), "cudaGraphLaunch");
        }
    }
    cudaGraph_t g = nullptr;
    if (!c->ck(cudaStreamBeginCapture(c->cap_stream, cudaStreamCaptureModeThreadLocal),
               "begin capture"))
        return false;
    const bool ok = enqueue_chunk(c, w0, styles, nb, out, c->cap_stream, last_level, false, in);
    const cudaError_t e = cudaStreamEndCapture(c->cap_stream, &g);
    if (!ok) {
        if (g) cudaGraphDestroy(g);
        return false;
    }
    if (!c->ck(e, "end capture")) return false;
    cudaGraphExec_t exec = nullptr;
    const cudaError_t ie = cudaGraphInstantiate(&exec, g, 0);
    cudaGraphDestroy(g);
    if (!c->ck(ie, "cudaGraphInstantiate")) return false;
    c->graphs.push_front({nb, styles, out, last_level, split, exec});
    while (c->graphs.size() > 32) {
        cudaGraphExecDestroy(c->graphs.back().exec);
        c->graphs.pop_back();
    }
    return c->ck(cudaGraphLaunch(exec, st), "cudaGraphLaunch");
}

// a kernel reports an expired bounded wait through the device flag
bool device_ok(tpmd_ctx *c) {
    int flag = 0;
    if (!c->ck(cudaMemcpy(&flag, c->err_flag, 4, cudaMemcpyDeviceToHost), "error flag D2H")) return false;
    if (flag) {
        cudaMemset(c->err_flag, 0, 4);
        return c->fail("a decoder kernel timed out waiting on its pipeline (results invalid)");
    }
    return true;
}

// Sub-batches of a host decode on a handle without the split schedule below
// (the FFMA path, fewer than four frames, or TPMD_SUBBATCH / TPMD_NO_SPLIT
// set). The frame copy (D2H) of one sub-batch
// overlaps the compute of the next, so only the last copy is exposed: whole
// max_batch chunks first, then the last chunk split into shrinking parts
// (ratio about 0.62, the copy/compute time ratio per frame with margin) so
// the exposed copy is small while each copy still hides under the next
// part's compute. TPMD_SUBBATCH=k forces equal parts of k frames.
std::vector<int64_t> sub_batch_plan(int64_t n, int64_t max_batch) {
    std::vector<int64_t> plan;
    if (const char *e = getenv("TPMD_SUBBATCH")) {
        const int64_t k = std::max<int64_t>(1, std::min<int64_t>(max_batch, atoll(e)));
        for (int64_t f = 0; f < n; f += k) plan.push_back(std::min<int64_t>(k, n - f));
        return plan;
    }
    const int64_t tail = std::min<int64_t>(n, max_batch);
    for (int64_t f = 0; f < n - tail; f += max_batch) plan.push_back(std::min<int64_t>(max_batch, n - tail - f));
    const int parts = tail >= 16 ? 4 : tail >= 4 ? 2 : 1;
    double w[4], wsum = 0.0;
    for (int i = 0; i < parts; i++) wsum += (w[i] = std::pow(0.62, i));
    int64_t left = tail;
    for (int i = 0; i < parts; i++) {
        int64_t k = i + 1 == parts ? left : std::max<int64_t>(1, std::llround(tail * w[i] / wsum));
        k = std::min<int64_t>(k, left - (parts - 1 - i));  // leave at least one frame per later part
        plan.push_back(k);
        left -= k;
    }
    return plan;
}

// The schedule of a host decode on a tcgen05 handle. A group's frames first
// run the levels up to r128 together; the r256 and r512 levels then run in
// parts, and each part's frames go to the host (second stream) while the
// next part, or the next group, computes. Splitting only the last two
// levels keeps the small, latency-bound early levels at the group's full
// batch. Measured on one B200 (50-frame chunk): the levels up to r128 cost
// about 0.30 ms + 36 us per frame, the r256 and r512 levels 43 us per frame
// and the copy of an f32 frame 58 us, so the copies, not the compute, set
// the pace of the tail levels. A chunk's last group therefore holds about a
// quarter of its frames in parts of about three: its copies start while
// the group computes and little is left to copy when the compute ends. The
// other group starts with a small part so that copying starts early.
// RGB24 frames copy in 14 us each, a third of their tail-level compute, so
// there the compute sets the pace: one group per chunk, most of its frames
// in the first part and three short parts after it, whose copies leave
// little to copy at the end.
struct group_plan {
    int64_t f0, n;               // the group's frames within the call
    std::vector<int64_t> parts;  // its tail-level parts, in order
};

std::vector<int64_t> equal_parts(int64_t total, int64_t k) {
    k = std::max<int64_t>(1, std::min(k, total));
    std::vector<int64_t> v;
    for (int64_t i = 0; i < k; i++) v.push_back(total / k + (i < total % k ? 1 : 0));
    return v;
}

std::vector<group_plan> split_plan(int64_t n, int64_t max_batch, bool rgb) {
    std::vector<group_plan> plan;
    auto lead = [](int64_t g, double first, int64_t k) {  // a small first part, then k equal ones
        const int64_t f = std::min<int64_t>(g, std::max<int64_t>(1, std::llround(first * g)));
        std::vector<int64_t> v{f};
        if (g > f)
            for (int64_t x : equal_parts(g - f, k)) v.push_back(x);
        return v;
    };
    int64_t f0 = 0;
    if (rgb) {
        for (; f0 < n; f0 += max_batch) {
            const int64_t g = std::min(max_batch, n - f0);
            plan.push_back({f0, g, lead(g, 0.58, 3)});
        }
        return plan;
    }
    for (; n - f0 > max_batch; f0 += max_batch) plan.push_back({f0, max_batch, lead(max_batch, 0.21, 3)});
    const int64_t m = n - f0;
    if (m < 16) {
        plan.push_back({f0, m, lead(m, 0.3, 2)});
    } else {
        const int64_t g2 = std::max<int64_t>(2, std::llround(0.24 * (double) m)), g1 = m - g2;
        plan.push_back({f0, g1, lead(g1, 0.21, 3)});
        plan.push_back({f0 + g1, g2, equal_parts(g2, std::max<int64_t>(1, std::llround((double) g2 / 3.0)))});
    }
    return plan;
}

bool ready(tpmd_ctx *c) {
    if (!c->wready) return c->fail("weights not prepared (tpmd_prepare)");
    if (!c->fready) return c->fail("feats not set (tpmd_set_feats)");
    if (!c->pready) return c->fail("feats projection missing (set the feats again)");
    return true;
}

}  // namespace

extern "C" {

int tpmd_decode_device(tpmd_ctx *c, const float *styles_dev, int64_t n, float *frames_dev,
                       void *stream) {
    nvtx_range range("tpmd_decode_device");
    if (!c) return -1;
    if (!styles_dev || !frames_dev || n < 1) return c->fail("tpmd_decode_device: bad argument"), -1;
    if (!ready(c)) return -1;
    if (!c->ck(cudaSetDevice(c->device), "cudaSetDevice")) return -1;
    cudaStream_t st = (cudaStream_t) stream;  // NULL: the legacy default stream
    const size_t fsz = (size_t) 3 * IMG * IMG;
    // after the handle's previous asynchronous decode, which may have run on
    // another stream (skipped inside a stream capture, which may not wait on
    // an event recorded outside it)
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (!c->ck(cudaStreamIsCapturing(st, &cs), "capture status") ||
        (cs == cudaStreamCaptureStatusNone && !c->ck(cudaStreamWaitEvent(st, c->ev_order, 0), "order wait")))
        return -1;
    for (int64_t f0 = 0; f0 < n; f0 += c->max_batch) {
        const int64_t nb = std::min<int64_t>(c->max_batch, n - f0);
        if (!run_chunk(c, styles_dev + f0 * STYLE_DIM, nb, frames_dev + f0 * fsz, st)) return -1;
    }
    if (cs == cudaStreamCaptureStatusNone && !c->ck(cudaEventRecord(c->ev_order, st), "order record")) return -1;
    return 0;
}

int64_t tpmd_kernel_launches(const tpmd_ctx *c, int64_t n) { return tpmd_kernel_launches_impl(c, n); }

int tpmd_decode_taps(tpmd_ctx *c, const float *style, int level, float *conv1, float *conv2,
                     float *flowmap, float *trunk, float *rgb) {
    if (!c) return -1;
    if (!style || level < 0 || level >= N_LEVELS) return c->fail("tpmd_decode_taps: bad argument"), -1;
    if (!ready(c)) return -1;
    if (!c->ck(cudaSetDevice(c->device), "cudaSetDevice") ||
        !c->ck(cudaStreamWaitEvent(c->stream, c->ev_order, 0), "order wait") ||
        !c->ck(cudaMemcpyAsync(c->styles_d[0], style, STYLE_DIM * 4, cudaMemcpyHostToDevice,
                               c->stream),
               "style H2D") ||
        !enqueue_chunk(c, ctx_ws(c), c->styles_d[0], 1, c->frames_d[0], c->stream, level, true) ||
        !c->ck(cudaStreamSynchronize(c->stream), "sync") || !device_ok(c))
        return -1;
    const int r = 8 << level, OC = ST_OC[level];
    const size_t n = (size_t) r * r * OC;
    // NHWC (f16 or f32) device buffer -> CHW f32 host
    auto fetch_act = [&](const void *dev, float *dst) {
        if (!dst) return true;
        std::vector<char> tmp(n * c->esz());
        if (!c->ck(cudaMemcpy(tmp.data(), dev, tmp.size(), cudaMemcpyDeviceToHost), "tap D2H"))
            return false;
        for (size_t p = 0; p < (size_t) r * r; p++)
            for (int ch = 0; ch < OC; ch++) {
                const size_t i = p * OC + ch;
                dst[(size_t) ch * r * r + p] = c->f16 ? __half2float(((const __half *) tmp.data())[i])
                                                      : ((const float *) tmp.data())[i];
            }
        return true;
    };
    auto fetch3 = [&](const float *dev, float *dst) {
        return !dst || c->ck(cudaMemcpy(dst, dev, (size_t) 3 * r * r * 4, cudaMemcpyDeviceToHost),
                             "tap D2H");
    };
    const bool last = level == N_LEVELS - 1;
    if (!fetch_act(c->actC, conv1) || !fetch_act(c->actA, conv2) ||
        (!last && !fetch3(c->sf[level & 1], flowmap)) || (!last && !fetch_act(c->actB, trunk)) ||
        !fetch3(last ? c->frames_d[0] : c->sk[level & 1], rgb))
        return -1;
    return 0;
}

int tpmd_profile_begin(tpmd_ctx *c) {
    if (!c) return -1;
    for (auto &r : c->prof) {
        cudaEventDestroy(r.a);
        cudaEventDestroy(r.b);
    }
    c->prof.clear();
    c->profiling = true;
    return 0;
}

int tpmd_profile_end(tpmd_ctx *c, char *json, size_t cap) {
    if (!c) return -1;
    c->profiling = false;
    std::map<std::string, std::pair<int64_t, double>> agg;
    std::vector<std::string> order;
    for (auto &r : c->prof) {
        float ms = 0.0f;
        if (!c->ck(cudaEventSynchronize(r.b), "event sync") ||
            !c->ck(cudaEventElapsedTime(&ms, r.a, r.b), "elapsed"))
            return -1;
        if (!agg.count(r.name)) order.push_back(r.name);
        agg[r.name].first += 1;
        agg[r.name].second += ms;
    }
    std::string out = "{";
    for (size_t i = 0; i < order.size(); i++) {
        char buf[160];
        snprintf(buf, sizeof buf, "%s\"%s\": [%lld, %.6f]", i ? ", " : "", order[i].c_str(),
                 (long long) agg[order[i]].first, agg[order[i]].second);
        out += buf;
    }
    out += "}";
    if (!json || out.size() + 1 > cap) return c->fail("tpmd_profile_end: buffer too small"), -1;
    memcpy(json, out.c_str(), out.size() + 1);
    return 0;
}

}  // extern "C"

namespace {

// The host decode loop: styles H2D, decode, (RGB24 conversion), frames D2H,
// each part's frame copy overlapping the next part's compute (split_plan on
// tcgen05 handles, else whole-decode sub-batches by sub_batch_plan).
int host_decode(tpmd_ctx *c, const float *styles, int64_t n, void *out, bool rgb, const char *who) {
    nvtx_range range(who);
    if (!c) return -1;
    if (!styles || !out || n < 1) return c->fail(std::string(who) + ": bad argument"), -1;
    if (!ready(c)) return -1;
    if (!c->ck(cudaSetDevice(c->device), "cudaSetDevice")) return -1;
    const size_t fsz = (size_t) 3 * IMG * IMG;
    const size_t osz = rgb ? fsz : fsz * 4;  // output bytes per frame
    // once anything is enqueued, a failure waits for both streams before
    // returning: no copy may still read the caller's styles or write its
    // frames after the call (the error message is the first failure's)
    auto bail = [&]() {
        cudaStreamSynchronize(c->copy_stream);
        cudaStreamSynchronize(c->stream);
        return -1;
    };
    // after the handle's previous asynchronous decode (tpmd_decode_device)
    if (!c->ck(cudaStreamWaitEvent(c->stream, c->ev_order, 0), "order wait")) return -1;
    if (c->use_tc && n >= 4 && !getenv("TPMD_SUBBATCH") && !getenv("TPMD_NO_SPLIT")) {
        // levels up to r128 per group, then the last two levels in parts
        constexpr int rs = 8 << (SPLIT_LEVEL - 1);
        const size_t tsz = (size_t) rs * rs * ST_OC[SPLIT_LEVEL - 1] * c->esz();  // r128 trunk bytes per frame
        const size_t ssz = (size_t) 3 * rs * rs;                                   // skip floats per frame
        const float *sf_in = c->sf[(SPLIT_LEVEL - 1) & 1], *sk_in = c->sk[(SPLIT_LEVEL - 1) & 1];
        int k = 0;
        for (const group_plan &g : split_plan(n, c->max_batch, rgb)) {
            if (!c->ck(cudaMemcpyAsync(c->styles_d[k], styles + g.f0 * STYLE_DIM,
                                       (size_t) g.n * STYLE_DIM * 4, cudaMemcpyHostToDevice, c->stream),
                       "styles H2D") ||
                !run_chunk(c, c->styles_d[k], g.n, nullptr, c->stream, SPLIT_LEVEL - 1) ||
                // staging buffer k is free once its previous frame copy finished
                !c->ck(cudaStreamWaitEvent(c->stream, c->ev_copied[k], 0), "wait"))
                return bail();
            int64_t p0 = 0;
            for (const int64_t np : g.parts) {
                const split_in in{(const char *) c->actB + p0 * tsz, sf_in + p0 * ssz, sk_in + p0 * ssz};
                float *fr = c->frames_d[k] + p0 * fsz;
                uint8_t *rg = c->rgb_d[k] + p0 * fsz;
                if (!run_chunk(c, nullptr, np, fr, c->stream, N_LEVELS - 1, &in, p0) ||
                    (rgb && !c->ck(launch_chw_to_rgb24(fr, np, (int64_t) IMG * IMG, rg, c->stream), "rgb24")) ||
                    !c->ck(cudaEventRecord(c->ev_done[k], c->stream), "record") ||
                    !c->ck(cudaStreamWaitEvent(c->copy_stream, c->ev_done[k], 0), "wait") ||
                    !c->ck(cudaMemcpyAsync((char *) out + (g.f0 + p0) * osz, rgb ? (const void *) rg : fr,
                                           (size_t) np * osz, cudaMemcpyDeviceToHost, c->copy_stream),
                           "frames D2H"))
                    return bail();
                p0 += np;
            }
            if (!c->ck(cudaEventRecord(c->ev_copied[k], c->copy_stream), "record")) return bail();
            k ^= 1;
        }
        if (!c->ck(cudaStreamSynchronize(c->copy_stream), "sync") ||
            !c->ck(cudaStreamSynchronize(c->stream), "sync"))
            return bail();
        return device_ok(c) ? 0 : -1;
    }
    const std::vector<int64_t> plan = sub_batch_plan(n, c->max_batch);
    int k = 0;
    int64_t f0 = 0;
    for (size_t i = 0; i < plan.size(); f0 += plan[i], i++, k ^= 1) {
        const int64_t nb = plan[i];
        // staging buffer k is free once its previous frame copy finished
        if (!c->ck(cudaStreamWaitEvent(c->stream, c->ev_copied[k], 0), "wait") ||
            !c->ck(cudaMemcpyAsync(c->styles_d[k], styles + f0 * STYLE_DIM,
                                   (size_t) nb * STYLE_DIM * 4, cudaMemcpyHostToDevice, c->stream),
                   "styles H2D") ||
            !run_chunk(c, c->styles_d[k], nb, c->frames_d[k], c->stream) ||
            (rgb && !c->ck(launch_chw_to_rgb24(c->frames_d[k], nb, (int64_t) IMG * IMG, c->rgb_d[k], c->stream),
                           "rgb24")) ||
            !c->ck(cudaEventRecord(c->ev_done[k], c->stream), "record") ||
            !c->ck(cudaStreamWaitEvent(c->copy_stream, c->ev_done[k], 0), "wait") ||
            !c->ck(cudaMemcpyAsync((char *) out + f0 * osz, rgb ? (const void *) c->rgb_d[k] : c->frames_d[k],
                                   (size_t) nb * osz, cudaMemcpyDeviceToHost, c->copy_stream),
                   "frames D2H") ||
            !c->ck(cudaEventRecord(c->ev_copied[k], c->copy_stream), "record"))
            return bail();
    }
    if (!c->ck(cudaStreamSynchronize(c->copy_stream), "sync") ||
        !c->ck(cudaStreamSynchronize(c->stream), "sync"))
        return bail();
    return device_ok(c) ? 0 : -1;
}

}  // namespace

extern "C" {

int tpmd_decode(tpmd_ctx *c, const float *styles, int64_t n, float *frames) {
    return host_decode(c, styles, n, frames, false, "tpmd_decode");
}

int64_t tpmd_decode_schedule(int64_t n, int64_t max_batch, int rgb, int64_t *out, int64_t cap) {
    if (n < 4 || max_batch < 1 || !out || cap < 0) return -1;
    int64_t w = 0;
    for (const group_plan &g : split_plan(n, max_batch, rgb != 0)) {
        if (w + 3 + (int64_t) g.parts.size() > cap) return -1;
        out[w++] = g.f0;
        out[w++] = g.n;
        out[w++] = (int64_t) g.parts.size();
        for (const int64_t p : g.parts) out[w++] = p;
    }
    return w;
}

int tpmd_decode_rgb24(tpmd_ctx *c, const float *styles, int64_t n, uint8_t *rgb) {
    return host_decode(c, styles, n, rgb, true, "tpmd_decode_rgb24");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Decoding without any allocation: the per-decode scratch lives in a static
// device array of this library instead of the handle's workspace.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t NOALLOC_BYTES = (size_t) 48 << 20;  // 48 MiB: one f16 frame's scratch
constexpr int NOALLOC_MAX_FRAMES = 1;

// Shared by every call on a device and kept between calls.
static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_BYTES];

std::mutex g_noalloc_mu;
void *g_noalloc_addr[64] = {nullptr};  // device address of the array, per device

// carve one frame's workspace out of the static array; false if it does not fit
bool noalloc_view(const tpmd_ctx *c, char *base, ws_view &w) {
    size_t a, b, cc;
    act_sizes(a, b, cc);
    const size_t skip = (size_t) 3 * 256 * 256;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        char *p = base + off;
        off = align256(off + bytes);
        return p;
    };
    w.err = (int *) take(256);  // first: tpmd_device_status reads it at offset 0
    w.s_all = (float *) take((size_t) c->S_TOT * 4);
    w.inv_den = (float *) take((size_t) c->D_TOT * 4);
    w.actA = take(a * c->esz());
    w.actB = take(b * c->esz());
    w.actC = take(cc * c->esz());
    for (int i = 0; i < 2; i++) w.sf[i] = (float *) take(skip * 4);
    for (int i = 0; i < 2; i++) w.sk[i] = (float *) take(skip * 4);
    w.timed = false;  // CUDA events would be allocations
    w.stall_ns = 0;
    return off <= NOALLOC_BYTES;
}

}  // namespace

extern "C" int tpmd_decode_noalloc(tpmd_ctx *c, const float *styles_dev, int64_t n,
                                   float *frames_dev, void *stream) {
    if (!c) return -1;
    if (!styles_dev || !frames_dev) return c->fail("tpmd_decode_noalloc: null pointer"), -1;
    if (n < 1 || n > NOALLOC_MAX_FRAMES)
        return c->fail("tpmd_decode_noalloc: n = " + std::to_string(n) +
                       " frames exceeds its static scratch (at most " +
                       std::to_string(NOALLOC_MAX_FRAMES) + " frame per call)"),
               -1;
    if (!c->f16)
        return c->fail("tpmd_decode_noalloc: the static scratch holds f16 activations only "
                       "(create the handle with TPMD_DTYPE_F16)"),
               -1;
    if (!ready(c)) return -1;
    if (c->device < 0 || c->device >= 64) return c->fail("tpmd_decode_noalloc: device index"), -1;
    if (!c->ck(cudaSetDevice(c->device), "cudaSetDevice")) return -1;
    char *base = nullptr;
    {
        // once per device, with that device current: the host-side name of the
        // array is not a device address, so ask the runtime for the real one
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        if (!g_noalloc_addr[c->device]) {
            void *p = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
            // the error word starts at zero; afterwards only tpmd_device_status clears it
            if (e == cudaSuccess) e = cudaMemset(p, 0, 256);
            if (e != cudaSuccess)
                return c->fail(std::string("tpmd_decode_noalloc: set-up: ") + cudaGetErrorString(e)), -1;
            g_noalloc_addr[c->device] = p;
        }
        base = (char *) g_noalloc_addr[c->device];
    }
    ws_view w;
    if (!noalloc_view(c, base, w)) return c->fail("tpmd_decode_noalloc: scratch layout too large"), -1;
    // every scratch buffer is written before it is read; the error word keeps
    // an expired wait until tpmd_device_status reads and clears it
    return enqueue_chunk(c, w, styles_dev, n, frames_dev, (cudaStream_t) stream) ? 0 : -1;
}

extern "C" int tpmd_device_status(tpmd_ctx *c, void *stream) {
    if (!c) return -1;
    if (!c->ck(cudaSetDevice(c->device), "cudaSetDevice") ||
        !c->ck(cudaStreamSynchronize((cudaStream_t) stream), "tpmd_device_status: stream"))
        return -1;
    void *na = nullptr;
    if (c->device >= 0 && c->device < 64) {
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        na = g_noalloc_addr[c->device];
    }
    int flag = 0, nflag = 0;
    if (!c->ck(cudaMemcpy(&flag, c->err_flag, 4, cudaMemcpyDeviceToHost), "tpmd_device_status: read") ||
        (na && !c->ck(cudaMemcpy(&nflag, na, 4, cudaMemcpyDeviceToHost), "tpmd_device_status: read")))
        return -1;
    if ((flag && !c->ck(cudaMemset(c->err_flag, 0, 4), "tpmd_device_status: clear")) ||
        (nflag && !c->ck(cudaMemset(na, 0, 4), "tpmd_device_status: clear")))
        return -1;
    if (flag || nflag)
        return c->fail("a decoder kernel timed out waiting on its pipeline (results invalid)"), -1;
    return 0;
}

extern "C" int tpmd_debug_expire_wait(tpmd_ctx *c, long long wait_ns) {
    if (!c) return -1;
    if (!c->use_tc) return c->fail("tpmd_debug_expire_wait: needs the tcgen05 path (TPMD_DTYPE_F16)"), -1;
    if (wait_ns < 1 || wait_ns > 2000000000ll)
        return c->fail("tpmd_debug_expire_wait: wait_ns must be in 1 .. 2e9"), -1;
    c->stall_ns = wait_ns;
    return 0;
}
