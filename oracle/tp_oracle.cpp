// CPU oracle for the motion decoder — TEST INFRASTRUCTURE ONLY (see
// tp_oracle.h). Each function names the reference lines it restates; paths are
// relative to the reference project root (patch:N = patches/ggml-tp-ops.patch
// line N).
#include "tp_oracle.h"

#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

namespace {

const int ST_IC[7] = {512, 512, 512, 512, 256, 128, 64};  // motion_dec.cpp:12
const int ST_OC[7] = {512, 512, 512, 256, 128, 64, 32};   // motion_dec.cpp:13

inline float h2f(uint16_t h) {
    _Float16 v;
    memcpy(&v, &h, 2);
    return (float) v;
}
inline uint16_t f2h(float f) {
    _Float16 v = (_Float16) f;  // round-to-nearest-even
    uint16_t h;
    memcpy(&h, &v, 2);
    return h;
}
inline float lrelu(float v, float s) { return v > 0.0f ? v : s * v; }
inline float r16(float v) { return (float) (_Float16) v; }
void round16(std::vector<float> &v) {
    for (auto &x : v) x = r16(x);
}

// One output row of a stride-1 2-D correlation for a block of `nb` output
// channels: acc[o][ox] += sum_{ic,ky,kx} w[o][ic][ky][kx] * x[ic][iy][ox+kx-pl]
// (iy = oy + ky - pt, zero outside the input). Cloned for AVX-512 / AVX2 so the
// oracle runs near the host's vector width wherever the library travels.
__attribute__((target_clones("arch=x86-64-v4", "default")))
void conv_row(const float *x, int IC, int IH, int IW, const float *w, int KH,
              int KW, int pt, int pl, int oy, int OW, int nb, float *acc,
              int accs) {
    for (int ic = 0; ic < IC; ic++) {
        for (int ky = 0; ky < KH; ky++) {
            const int iy = oy + ky - pt;
            if (iy < 0 || iy >= IH) continue;
            const float *row = x + ((size_t) ic * IH + iy) * IW;
            for (int kx = 0; kx < KW; kx++) {
                const int sh = kx - pl;
                const int lo = std::max(0, -sh), hi = std::min(OW, IW - sh);
                for (int o = 0; o < nb; o++) {
                    const float wv = w[(((size_t) o * IC + ic) * KH + ky) * KW + kx];
                    float *a = acc + (size_t) o * accs;
                    for (int ox = lo; ox < hi; ox++) a[ox] += wv * row[ox + sh];
                }
            }
        }
    }
}

// Register-blocked form of conv_row for 8 output channels and 16 output
// columns: the 8 x 16 sums stay in eight vector registers while (ic, ky, kx) runs, and the
// input comes from a copy padded by pl columns on the left and enough on the
// right (xpad rows of width PW), so no column test sits in the inner loop.
// Each output is still summed in (ic, ky, kx) order.
typedef float v16f __attribute__((vector_size(64)));
__attribute__((target_clones("arch=x86-64-v4", "default")))
void conv_tile8x16(const float *xpad, int IC, int IH, int PW, const float *w, int KH, int KW,
                   int pt, int oy, int ox0, float *y, int OH, int OW) {
    v16f a0 = {}, a1 = {}, a2 = {}, a3 = {}, a4 = {}, a5 = {}, a6 = {}, a7 = {};
    const size_t ws = (size_t) IC * KH * KW;  // weight stride between output channels
    for (int ic = 0; ic < IC; ic++) {
        for (int ky = 0; ky < KH; ky++) {
            const int iy = oy + ky - pt;
            if (iy < 0 || iy >= IH) continue;
            const float *row = xpad + ((size_t) ic * IH + iy) * PW + ox0;
            const float *wk = w + ((size_t) ic * KH + ky) * KW;
            for (int kx = 0; kx < KW; kx++) {
                v16f xv;
                memcpy(&xv, row + kx, sizeof xv);
                a0 += wk[kx] * xv;
                a1 += wk[ws + kx] * xv;
                a2 += wk[2 * ws + kx] * xv;
                a3 += wk[3 * ws + kx] * xv;
                a4 += wk[4 * ws + kx] * xv;
                a5 += wk[5 * ws + kx] * xv;
                a6 += wk[6 * ws + kx] * xv;
                a7 += wk[7 * ws + kx] * xv;
            }
        }
    }
    const v16f *acc[8] = {&a0, &a1, &a2, &a3, &a4, &a5, &a6, &a7};
    for (int o = 0; o < 8; o++) memcpy(y + ((size_t) o * OH + oy) * OW + ox0, acc[o], sizeof(v16f));
}

// y[OC][OH][OW] = corr2d(x[IC][IH][IW], w[OC][IC][KH][KW]), stride 1, top/left
// padding pt/pl (zeros), output size given (the bottom/right padding follows).
// Stands in for ggml_conv_2d_direct as used by src/motion_dec.cpp:597-632.
void conv2d(const float *x, int IC, int IH, int IW, const float *w, int OC, int KH,
            int KW, int pt, int pl, int OH, int OW, float *y) {
    const int OB = 8;
    const int nob = (OC + OB - 1) / OB;
    // zero-padded copy of the input for the 8 x 16 tiles: columns -pl .. OW+KW
    const int PW = OW + KW + 16;
    std::vector<float> xpad;
    const bool tiles = OW >= 16;
    if (tiles) {
        xpad.assign((size_t) IC * IH * PW, 0.0f);
#pragma omp parallel for schedule(static)
        for (int r = 0; r < IC * IH; r++)
            for (int c = 0; c < IW; c++) {
                const int pc = c + pl;
                if (pc >= 0 && pc < PW) xpad[(size_t) r * PW + pc] = x[(size_t) r * IW + c];
            }
    }
    const int ntile = tiles ? OW / 16 : 0;
#pragma omp parallel
    {
        std::vector<float> acc((size_t) OB * OW);
#pragma omp for collapse(2) schedule(dynamic, 4)
        for (int ob = 0; ob < nob; ob++) {
            for (int oy = 0; oy < OH; oy++) {
                const int o0 = ob * OB, nb = std::min(OB, OC - o0);
                if (nb == OB && ntile > 0) {
                    for (int t = 0; t < ntile; t++)
                        conv_tile8x16(xpad.data(), IC, IH, PW, w + (size_t) o0 * IC * KH * KW, KH, KW, pt, oy,
                                      16 * t, y + (size_t) o0 * OH * OW, OH, OW);
                    if (ntile * 16 == OW) continue;
                }
                // channel-block remainder, narrow maps and the last columns: row form
                std::fill(acc.begin(), acc.end(), 0.0f);
                conv_row(x, IC, IH, IW, w + (size_t) o0 * IC * KH * KW, KH, KW, pt, pl,
                         oy, OW, nb, acc.data(), OW);
                const int c0 = (nb == OB) ? ntile * 16 : 0;
                for (int o = 0; o < nb; o++)
                    memcpy(y + ((size_t) (o0 + o) * OH + oy) * OW + c0,
                           acc.data() + (size_t) o * OW + c0, (size_t) (OW - c0) * 4);
            }
        }
    }
}

std::map<std::string, int64_t> expected_tensors() {
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
    for (int j = 0; j < 7; j++) {
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

}  // namespace

extern "C" {

// ---------------------------------------------------------------------------
// patched ops
// ---------------------------------------------------------------------------

// torch grid_sample (bilinear, zeros, align_corners=false) over a channel-last
// map; patch:319-369 (CPU) / patch:688-718 (CUDA). fx = (gx+1)/2*W - 1/2 with
// the final multiply-add fused, taps k = 0..3 at (x0 + (k&1), y0 + (k>>1)),
// out-of-range taps skipped, accumulation in tap order with fused multiply-add.
void orc_bilinear_gather(const void *feat, int feat_f16, int C, int W, int H,
                         const float *grid, int64_t N, int planar, int sp,
                         float *dst) {
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; n++) {
        const float gx = planar ? grid[n] : grid[2 * n + 0];
        const float gy = planar ? grid[N + n] : grid[2 * n + 1];
        const float fx = fmaf((gx + 1.0f) * 0.5f, (float) W, -0.5f);
        const float fy = fmaf((gy + 1.0f) * 0.5f, (float) H, -0.5f);
        const int64_t x0 = (int64_t) floorf(fx), y0 = (int64_t) floorf(fy);
        const float wx = fx - (float) x0, wy = fy - (float) y0;
        float *d = dst + (sp ? n : (int64_t) C * n);
        const int64_t ds = sp ? N : 1;
        for (int c = 0; c < C; c++) d[c * ds] = 0.0f;
        for (int k = 0; k < 4; k++) {
            const int64_t cx = x0 + (k & 1), cy = y0 + (k >> 1);
            if (cx < 0 || cx >= W || cy < 0 || cy >= H) continue;
            const float wgt = ((k & 1) ? wx : 1.0f - wx) * ((k >> 1) ? wy : 1.0f - wy);
            const int64_t row = cy * W + cx;
            if (feat_f16) {
                const uint16_t *f = (const uint16_t *) feat + (int64_t) C * row;
                for (int c = 0; c < C; c++) d[c * ds] = fmaf(wgt, h2f(f[c]), d[c * ds]);
            } else {
                const float *f = (const float *) feat + (int64_t) C * row;
                for (int c = 0; c < C; c++) d[c * ds] = fmaf(wgt, f[c], d[c * ds]);
            }
        }
    }
}

// channels-first im2col, patch:201-307 (CPU) / patch:830-861 (CUDA): source
// [IC, IW, IH, N] (ic fastest), dst [IC*KW*KH, OW, OH, N] with row
// r = ic + IC*(kw + KW*kh), zero outside the source.
void orc_im2col_cf(const float *src, int IC, int IW, int IH, int N, int KW, int KH,
                   int s0, int s1, int p0, int p1, int d0, int d1, void *dst,
                   int dst_f16) {
    const int64_t OW = (IW + 2 * p0 - d0 * (KW - 1) - 1) / s0 + 1;
    const int64_t OH = (IH + 2 * p1 - d1 * (KH - 1) - 1) / s1 + 1;
    const int64_t R = (int64_t) IC * KW * KH;
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t in = 0; in < N; in++) {
        for (int64_t oh = 0; oh < OH; oh++) {
            for (int64_t ow = 0; ow < OW; ow++) {
                const int64_t base = ((in * OH + oh) * OW + ow) * R;
                const float *sb = src + in * (int64_t) IC * IW * IH;
                for (int kh = 0; kh < KH; kh++) {
                    for (int kw = 0; kw < KW; kw++) {
                        const int64_t iw = ow * s0 + kw * d0 - p0;
                        const int64_t ih = oh * s1 + kh * d1 - p1;
                        const bool in_b = iw >= 0 && iw < IW && ih >= 0 && ih < IH;
                        for (int ic = 0; ic < IC; ic++) {
                            const int64_t r = ic + (int64_t) IC * (kw + KW * kh);
                            const float v = in_b ? sb[ic + (int64_t) IC * (iw + IW * ih)] : 0.0f;
                            if (dst_f16)
                                ((uint16_t *) dst)[base + r] = f2h(v);
                            else
                                ((float *) dst)[base + r] = v;
                        }
                    }
                }
            }
        }
    }
}

// y = leaky_relu(x + bias, slope), bias along ggml dim `axis` (0 or 2);
// patch:376-430.
void orc_bias_lrelu(const float *x, const float *bias, const int64_t *ne, int axis,
                    float slope, float *y) {
    const int64_t n = ne[0] * ne[1] * ne[2] * ne[3];
    const int64_t C = ne[axis], d01 = ne[0] * ne[1];
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) {
        const int64_t c = axis == 0 ? i % C : (i / d01) % C;
        y[i] = lrelu(x[i] + bias[c], slope);
    }
}

// spatial sub-pixel interleave + bias + lrelu, patch:435-482:
// dst[2n+bx, 2m+by, o] = lrelu(g{by}[n, m, o + OC*bx] + bias[o]).
void orc_subpix_lrelu(const float *g0, const float *g1, const float *bias, int W,
                      int H, int OC, float slope, float *y) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int o = 0; o < OC; o++) {
        for (int Y = 0; Y < 2 * H; Y++) {
            const float *g = (Y & 1) ? g1 : g0;
            const int m = Y >> 1;
            for (int X = 0; X < 2 * W; X++) {
                const int nn = X >> 1, bx = X & 1;
                const float v = g[nn + (int64_t) W * (m + (int64_t) H * (o + OC * bx))] + bias[o];
                y[X + 2 * (int64_t) W * (Y + 2 * (int64_t) H * o)] = lrelu(v, slope);
            }
        }
    }
}

// channel-last sub-pixel interleave, patch:488-530:
// dst[o, (2n+bx) + 2W(2m+by), b] = lrelu(y4[o + OC*(2by+bx), n + W*m, b] + bias[o]).
void orc_subpix_lrelu_cl(const float *y4, const float *bias, int OC, int64_t N,
                         int64_t B, int W, float slope, float *y) {
    const int64_t W2 = 2 * (int64_t) W;
    const int64_t npix = 4 * N * B;
#pragma omp parallel for schedule(static)
    for (int64_t p = 0; p < npix; p++) {
        const int64_t nn = p % (4 * N), bb = p / (4 * N);
        const int64_t X = nn % W2, Y = nn / W2;
        const int64_t k = (Y & 1) * 2 + (X & 1);
        const float *s = y4 + OC * k + 4 * (int64_t) OC * ((X >> 1) + W * (Y >> 1) + N * bb);
        for (int o = 0; o < OC; o++) y[(int64_t) OC * p + o] = lrelu(s[o] + bias[o], slope);
    }
}

// upfirdn2d(up=2, pad=(2,1)) with a 4x4 FIR, patch:535-572:
// y[X,Y] = sum_{j,i} zstuff(x)[X+i-2, Y+j-2] * k4[i + 4j].
void orc_upfirdn2x(const float *x, const float *k4, int W, int H, int64_t CB,
                   float *y) {
    const int64_t n_tot = 4 * (int64_t) W * H * CB;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n_tot; i++) {
        const int64_t X = i % (2 * W), Y = (i / (2 * W)) % (2 * H);
        const int64_t cb = i / (4 * (int64_t) W * H);
        const float *xp = x + (int64_t) W * H * cb;
        float acc = 0.0f;
        for (int j = 0; j < 4; j++) {
            const int64_t vy = Y + j - 2;
            if (vy < 0 || vy >= 2 * H || (vy & 1)) continue;
            for (int ii = 0; ii < 4; ii++) {
                const int64_t vx = X + ii - 2;
                if (vx < 0 || vx >= 2 * W || (vx & 1)) continue;
                acc = fmaf(xp[(vx >> 1) + W * (vy >> 1)], k4[ii + 4 * j], acc);
            }
        }
        y[i] = acc;
    }
}

// upfirdn2d(up=1, pad=(p0,p1)) with a 4x4 FIR (the Blur module,
// src/ops_common.h:39-43: pad_ext then depthwise correlation, no flip):
// x [C][H][W] -> y [C][H+p0+p1-3][W+p0+p1-3].
void orc_blur(const float *x, const float *k4, int W, int H, int64_t C, int p0, int p1,
              float *y) {
    const int OW = W + p0 + p1 - 3, OH = H + p0 + p1 - 3;
#pragma omp parallel for schedule(static)
    for (int64_t c = 0; c < C; c++)
        for (int Y = 0; Y < OH; Y++)
            for (int X = 0; X < OW; X++) {
                float acc = 0.0f;
                for (int a = 0; a < 4; a++) {
                    const int sy = Y + a - p0;
                    if (sy < 0 || sy >= H) continue;
                    for (int b = 0; b < 4; b++) {
                        const int sx = X + b - p0;
                        if (sx < 0 || sx >= W) continue;
                        acc += k4[a * 4 + b] * x[((size_t) c * H + sy) * W + sx];
                    }
                }
                y[((size_t) c * OH + Y) * OW + X] = acc;
            }
}

// channel-last -> spatial transpose times the mask, patch:578-601.
void orc_clsp_mul(const float *cl, const float *m, int C, int64_t N, float *y) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int c = 0; c < C; c++)
        for (int64_t n = 0; n < N; n++) y[n + N * c] = cl[c + (int64_t) C * n] * m[n];
}

// transpose + blend, patch:603-626: y = cl^T*m + out*(1-m).
void orc_clsp_lerp(const float *cl, const float *m, const float *o, int C, int64_t N,
                   float *y) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int c = 0; c < C; c++)
        for (int64_t n = 0; n < N; n++) {
            const int64_t i = n + N * c;
            const float a = cl[c + (int64_t) C * n] * m[n];
            const float b = o[i] * (1.0f - m[n]);
            y[i] = a + b;
        }
}

// flow head, patch:632-657: planar (tanh(f0)+xs0, tanh(f1)+xs1, sigmoid(f2)).
void orc_flow_grid(const float *fl, const float *xs, int64_t N, float *y) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < 3 * N; i++) {
        const int64_t pln = i / N, n = i % N;
        y[i] = pln == 2 ? 1.0f / (1.0f + expf(-fl[2 * N + n]))
                        : tanhf(fl[pln * N + n]) + xs[pln * N + n];
    }
}

// ---------------------------------------------------------------------------
// load-time scale folding: src/motion_enc.cpp:14-45
// ---------------------------------------------------------------------------
double orc_scale_for(const char *cname, const int64_t *ne) {
    const std::string name = cname;
    const double SQRT2 = 1.4142135623730951;
    auto ends = [&](const char *s) {
        const size_t n = strlen(s);
        return name.size() >= n && name.compare(name.size() - n, n, s) == 0;
    };
    auto starts = [&](const char *s) { return name.rfind(s, 0) == 0; };
    if (name == "enc.net_app.convs.0.1.bias" || ends(".conv1.1.bias") ||
        ends(".activate.bias") || (starts("dec.to_rgbs.") && ends(".conv.1.bias")))
        return SQRT2;
    if (!ends(".weight")) return 1.0;
    if (starts("dec.direction")) return 1.0;
    if (ends("noise.weight")) return 1.0;
    if (ends("modulation.weight")) return 1.0 / sqrt((double) ne[0]);
    if (starts("enc.fc.")) return 1.0 / sqrt((double) ne[0]);
    const double conv = 1.0 / sqrt((double) (ne[0] * ne[1] * ne[2]));
    if (name == "enc.net_app.convs.0.0.weight" || ends(".conv1.0.weight")) return conv * SQRT2;
    if (ends(".conv2.1.weight")) return conv;
    if (ends(".skip.1.weight")) return conv / SQRT2;
    if (name == "enc.net_app.convs.8.weight") return conv;
    if (starts("dec.to_rgbs.") && ends(".conv.0.weight")) return conv * SQRT2;
    if (ends(".conv.weight")) return conv;
    return 1.0;
}

// ---------------------------------------------------------------------------
// derived weights: src/motion_dec.cpp:108-120 (S_aug), :144-191 (tsubcf)
// ---------------------------------------------------------------------------
void orc_saug(const float *W, int IC, int OC, float *saug) {
    for (int o = 0; o < OC; o++) {
        for (int i = 0; i < IC; i++) {
            double s = 0;
            const float *pw = W + ((size_t) o * IC + i) * 9;
            for (int k = 0; k < 9; k++) s += (double) pw[k] * pw[k];
            saug[(size_t) o * (IC + 1) + i] = (float) (s * 0.5);
        }
        saug[(size_t) o * (IC + 1) + IC] = 0.5e-8f;
    }
}

// conv_transpose(3x3, stride 2) followed by the 4x4 blur (pad 1,1) equals, per
// output parity class (by, bx), a 3x3 pad-1 correlation of the input with
// T[ty][tx] = sum_{cy,cx} V[cy][cx] * K[1+2ty-by-cy][1+2tx-bx-cx]
// (V = spatially flipped weight, K = blur kernel, terms outside K dropped).
void orc_tsubcf(const float *W, const float *K, int IC, int OC, float *tsub) {
    const size_t R = (size_t) IC * 9;
#pragma omp parallel for schedule(static)
    for (int o = 0; o < OC; o++) {
        for (int i = 0; i < IC; i++) {
            const float *pw = W + ((size_t) o * IC + i) * 9;
            for (int by = 0; by < 2; by++)
                for (int bx = 0; bx < 2; bx++) {
                    float *dstc = tsub + (size_t) ((by * 2 + bx) * OC + o) * R;
                    for (int ty = 0; ty < 3; ty++)
                        for (int tx = 0; tx < 3; tx++) {
                            double acc = 0;
                            for (int cy = 0; cy < 3; cy++) {
                                const int ay = 1 + 2 * ty - by - cy;
                                if (ay < 0 || ay > 3) continue;
                                for (int cx = 0; cx < 3; cx++) {
                                    const int ax = 1 + 2 * tx - bx - cx;
                                    if (ax < 0 || ax > 3) continue;
                                    const float v = pw[(2 - cy) * 3 + (2 - cx)];
                                    acc += (double) v * (double) K[ay * 4 + ax];
                                }
                            }
                            dstc[i + (size_t) IC * (tx + 3 * ty)] = (float) acc;
                        }
                }
        }
    }
}

void orc_set_threads(int n) {
    if (n > 0) omp_set_num_threads(n);
}
int orc_get_threads(void) { return omp_get_max_threads(); }

}  // extern "C"

// ---------------------------------------------------------------------------
// decoder
// ---------------------------------------------------------------------------
struct orc_dec {
    std::map<std::string, int64_t> spec = expected_tensors();
    std::map<std::string, std::vector<float>> t;
    std::vector<float> feat[7];
    std::map<std::string, std::vector<float>> saug, tsub;
    std::map<std::string, std::vector<float>> taps;
    bool prepared = false;
    std::string err;

    const std::vector<float> &get(const std::string &n) const { return t.at(n); }

    // s = Wmod * latent + bmod (src/motion_dec.cpp:267-272). f16: the
    // reference keeps the modulation weights f16 in its f16 mode (every
    // file-f16 tensor of >= 4096 elements, src/gguf_load.cpp:149-153), and a
    // GEMM with f16 weights rounds its other operand to f16 too
    std::vector<float> style_of(const std::string &base, const float *lat, bool f16 = false) const {
        const std::vector<float> &Wm = get(base + ".modulation.weight");
        const std::vector<float> &bm = get(base + ".modulation.bias");
        const int IC = (int) bm.size();
        std::vector<float> s((size_t) IC);
        for (int i = 0; i < IC; i++) {
            double a = 0;
            const float *w = Wm.data() + (size_t) i * 512;
            for (int k = 0; k < 512; k++)
                a += f16 ? (double) r16(w[k]) * r16(lat[k]) : (double) w[k] * lat[k];
            s[(size_t) i] = (float) a + bm[(size_t) i];
        }
        return s;
    }
    // den = sqrt(S_aug [s^2; 1]) (src/motion_dec.cpp:275-280)
    std::vector<float> demod_den(const std::string &wname, const std::vector<float> &s) const {
        const std::vector<float> &sa = saug.at(wname);
        const int IC = (int) s.size();
        const int OC = (int) (sa.size() / (IC + 1));
        std::vector<float> den((size_t) OC);
        for (int o = 0; o < OC; o++) {
            const float *r = sa.data() + (size_t) o * (IC + 1);
            double a = 0;
            for (int i = 0; i < IC; i++) {
                const float s2 = s[(size_t) i] * s[(size_t) i];
                a += (double) r[i] * s2;
            }
            a += (double) r[IC];
            den[(size_t) o] = sqrtf((float) a);
        }
        return den;
    }
    void tap(bool keep, const std::string &name, const float *p, size_t n) {
        if (keep) taps[name].assign(p, p + n);
    }
};

namespace {

// modulated dense 3x3 conv, map-side style (src/motion_dec.cpp:597-608):
// lrelu(conv(x*s, W)/den + bias)
// The reference's f16 fast graph (ORC_F16_FOLD) multiplies the style and
// 1/den into the f16 weights when the map is larger than the weights,
// 4|W| < 2 N (IC + OC') (src/motion_dec.cpp:322-337), and always at the
// spatial stages (maps >= 256, src/motion_dec.cpp:452-466); the folded
// weights are rounded to f16 and the unstyled map is rounded to f16 as the
// GEMM's other operand. Otherwise it multiplies the map (rounded to f16 after
// the style) and divides by den after the GEMM. conv1 (4x4) is map side.
bool ref_folds(int64_t wsz, int64_t N, int64_t IC, int64_t OCp, int out_map) {
    if (out_map >= 256) return true;
    if (out_map <= 4) return false;
    return 4 * wsz < 2 * N * (IC + OCp);
}

std::vector<float> styled_conv_exact(const orc_dec &d, const std::vector<float> &x, int IC,
                                     int Hh, const std::string &base, const float *lat,
                                     int flags) {
    const bool fold16 = (flags & ORC_F16_FOLD) != 0;
    const std::vector<float> s = d.style_of(base + ".conv", lat, fold16);
    const std::vector<float> den = d.demod_den(base + ".conv.weight", s);
    if (fold16) {
        const std::vector<float> &W0 = d.get(base + ".conv.weight");
        const std::vector<float> &ab = d.get(base + ".activate.bias");
        const int OC = (int) ab.size();
        const size_t P = (size_t) Hh * Hh;
        const bool fold = ref_folds((int64_t) 9 * IC * OC, (int64_t) P, IC, OC, Hh);
        std::vector<float> W(W0.size()), xs(x.size());
        for (int o = 0; o < OC; o++)
            for (int i = 0; i < IC; i++)
                for (int k = 0; k < 9; k++) {
                    const size_t q = ((size_t) o * IC + i) * 9 + k;
                    W[q] = fold ? r16(r16(W0[q]) * s[(size_t) i] / den[(size_t) o]) : r16(W0[q]);
                }
        // conv1's constant input is itself stored f16; the styled map is the
        // product of f16 operands rounded to f16 (an f16 elementwise result)
        const bool f16_input = Hh == 4;
        for (int i = 0; i < IC; i++)
            for (size_t p = 0; p < P; p++) {
                const float v = f16_input ? r16(x[i * P + p]) : x[i * P + p];
                xs[i * P + p] = fold ? r16(v) : r16(v * s[(size_t) i]);
            }
        std::vector<float> y((size_t) OC * P);
        conv2d(xs.data(), IC, Hh, Hh, W.data(), OC, 3, 3, 1, 1, Hh, Hh, y.data());
#pragma omp parallel for schedule(static)
        for (int o = 0; o < OC; o++)
            for (size_t p = 0; p < P; p++) {
                const float v = fold ? y[o * P + p] : y[o * P + p] / den[(size_t) o];
                y[o * P + p] = lrelu(v + ab[(size_t) o], 0.2f);
            }
        return y;
    }
    std::vector<float> Wr;
    if (flags & ORC_F16_WEIGHTS) {
        Wr = d.get(base + ".conv.weight");
        round16(Wr);
    }
    const std::vector<float> &W = (flags & ORC_F16_WEIGHTS) ? Wr : d.get(base + ".conv.weight");
    const std::vector<float> &ab = d.get(base + ".activate.bias");
    const int OC = (int) ab.size();
    const size_t P = (size_t) Hh * Hh;
    std::vector<float> xs(x.size());
    for (int i = 0; i < IC; i++)
        for (size_t p = 0; p < P; p++) xs[i * P + p] = x[i * P + p] * s[(size_t) i];
    if (flags & ORC_F16_ACTS) round16(xs);
    std::vector<float> y((size_t) OC * P);
    conv2d(xs.data(), IC, Hh, Hh, W.data(), OC, 3, 3, 1, 1, Hh, Hh, y.data());
#pragma omp parallel for schedule(static)
    for (int o = 0; o < OC; o++)
        for (size_t p = 0; p < P; p++) {
            const float v = y[o * P + p] / den[(size_t) o];
            y[o * P + p] = lrelu(v + ab[(size_t) o], 0.2f);
        }
    return y;
}

// upsampling modulated conv.
// mode 0 (src/motion_dec.cpp:609-627): zero-stuff x*s, pad (2,1), correlate
// with the flipped weight, /den, blur pad (1,1), lrelu(+bias).
// mode 1 (src/motion_dec.cpp:397-433): the composed sub-pixel kernel (tsubcf)
// as one 3x3 pad-1 conv with 4*OC outputs, /den per class, sub-pixel shuffle,
// lrelu(+bias).
std::vector<float> styled_conv_up(const orc_dec &d, const std::vector<float> &x, int IC,
                                  int Hh, const std::string &base, const float *lat,
                                  int mode, int flags) {
    const bool fold16 = mode == 1 && (flags & ORC_F16_FOLD) != 0;
    const std::vector<float> s = d.style_of(base + ".conv", lat, fold16);
    const std::vector<float> den = d.demod_den(base + ".conv.weight", s);
    const std::vector<float> &W = d.get(base + ".conv.weight");
    const std::vector<float> &ab = d.get(base + ".activate.bias");
    const std::vector<float> &K = d.get(base + ".conv.blur.kernel");
    const int OC = (int) ab.size();
    const int H2 = 2 * Hh;
    const size_t P = (size_t) Hh * Hh;
    std::vector<float> out((size_t) OC * H2 * H2);
    if (mode == 0) {
        const int ZP = H2 + 3;  // zero-stuffed 2H, padded 2 before and 1 after
        std::vector<float> zs((size_t) IC * ZP * ZP, 0.0f);
        for (int i = 0; i < IC; i++)
            for (int yy = 0; yy < Hh; yy++)
                for (int xx = 0; xx < Hh; xx++)
                    zs[((size_t) i * ZP + 2 * yy + 2) * ZP + 2 * xx + 2] =
                        (flags & ORC_F16_ACTS) ? r16(x[i * P + (size_t) yy * Hh + xx] * s[(size_t) i])
                                               : x[i * P + (size_t) yy * Hh + xx] * s[(size_t) i];
        std::vector<float> wf(W.size());
        for (int o = 0; o < OC; o++)
            for (int i = 0; i < IC; i++)
                for (int a = 0; a < 3; a++)
                    for (int b = 0; b < 3; b++)
                        wf[(((size_t) o * IC + i) * 3 + a) * 3 + b] =
                            W[(((size_t) o * IC + i) * 3 + (2 - a)) * 3 + (2 - b)];
        if (flags & ORC_F16_WEIGHTS) round16(wf);
        const int TO = H2 + 1;  // conv_transpose output size 2H+1
        std::vector<float> y((size_t) OC * TO * TO);
        conv2d(zs.data(), IC, ZP, ZP, wf.data(), OC, 3, 3, 0, 0, TO, TO, y.data());
        // /den, then Blur with pad (1,1) (src/motion_dec.cpp:623-625)
#pragma omp parallel for schedule(static)
        for (int o = 0; o < OC; o++) {
            float *yo = y.data() + (size_t) o * TO * TO;
            for (size_t q = 0; q < (size_t) TO * TO; q++) yo[q] = yo[q] / den[(size_t) o];
        }
        orc_blur(y.data(), K.data(), TO, TO, OC, 1, 1, out.data());
#pragma omp parallel for schedule(static)
        for (int o = 0; o < OC; o++)
            for (size_t q = 0; q < (size_t) H2 * H2; q++) {
                float &v = out[(size_t) o * H2 * H2 + q];
                v = lrelu(v + ab[(size_t) o], 0.2f);
            }
    } else {
        const std::vector<float> &T = d.tsub.at(base + ".conv.weight");
        const size_t R = (size_t) IC * 9;
        // spatial [4OC][IC][3][3] view of the cf-ordered rows
        std::vector<float> w4((size_t) 4 * OC * R);
        for (int q = 0; q < 4 * OC; q++)
            for (int i = 0; i < IC; i++)
                for (int kh = 0; kh < 3; kh++)
                    for (int kw = 0; kw < 3; kw++)
                        w4[(((size_t) q * IC + i) * 3 + kh) * 3 + kw] =
                            T[(size_t) q * R + i + (size_t) IC * (kw + 3 * kh)];
        // f16 fast graph: fold (style, 1/den) into the f16 composed weights
        // or multiply the map, by the reference's rule (see ref_folds)
        const bool fold = fold16 && ref_folds((int64_t) 9 * IC * 4 * OC, (int64_t) P, IC, 4 * OC, H2);
        if (fold16)
            for (int q = 0; q < 4 * OC; q++)
                for (int i = 0; i < IC; i++)
                    for (int k = 0; k < 9; k++) {
                        float &v = w4[((size_t) q * IC + i) * 9 + k];
                        v = fold ? r16(r16(v) * s[(size_t) i] / den[(size_t) (q % OC)]) : r16(v);
                    }
        else if (flags & ORC_F16_WEIGHTS)
            round16(w4);
        std::vector<float> xs(x.size());
        for (int i = 0; i < IC; i++)
            for (size_t p = 0; p < P; p++) xs[i * P + p] = fold ? x[i * P + p] : x[i * P + p] * s[(size_t) i];
        if (flags & (ORC_F16_ACTS | ORC_F16_FOLD)) round16(xs);
        std::vector<float> y4((size_t) 4 * OC * P);
        conv2d(xs.data(), IC, Hh, Hh, w4.data(), 4 * OC, 3, 3, 1, 1, Hh, Hh, y4.data());
#pragma omp parallel for schedule(static)
        for (int o = 0; o < OC; o++)
            for (int Y = 0; Y < H2; Y++)
                for (int X = 0; X < H2; X++) {
                    const int k = (Y & 1) * 2 + (X & 1);
                    const float a = y4[((size_t) (k * OC + o)) * P + (size_t) (Y >> 1) * Hh + (X >> 1)];
                    const float v = fold ? a : a / den[(size_t) o];
                    out[((size_t) o * H2 + Y) * H2 + X] = lrelu(v + ab[(size_t) o], 0.2f);
                }
    }
    return out;
}

}  // namespace

extern "C" {

orc_dec *orc_dec_create(void) { return new orc_dec(); }
void orc_dec_destroy(orc_dec *d) { delete d; }
const char *orc_dec_error(const orc_dec *d) { return d ? d->err.c_str() : "null decoder"; }

int orc_dec_set(orc_dec *d, const char *name, const float *data, int64_t n) {
    auto it = d->spec.find(name);
    if (it == d->spec.end()) {
        d->err = std::string("unknown tensor ") + name;
        return -1;
    }
    if (it->second != n) {
        d->err = std::string(name) + ": size mismatch";
        return -1;
    }
    d->t[name].assign(data, data + n);
    d->prepared = false;
    return 0;
}

int orc_dec_set_feat(orc_dec *d, int j, const float *feat, int64_t n) {
    if (j < 0 || j > 6) {
        d->err = "feat level out of range";
        return -1;
    }
    const int r = 8 << j;
    if (n != (int64_t) ST_OC[j] * r * r) {
        d->err = "feat size mismatch";
        return -1;
    }
    d->feat[j].assign(feat, feat + n);
    return 0;
}

int orc_dec_prepare(orc_dec *d) {
    for (auto &kv : d->spec)
        if (!d->t.count(kv.first)) {
            d->err = "missing tensor " + kv.first;
            return -1;
        }
    std::vector<std::string> convs = {"dec.conv1.conv.weight"};
    for (int i = 0; i < 14; i++) convs.push_back("dec.convs." + std::to_string(i) + ".conv.weight");
    for (size_t c = 0; c < convs.size(); c++) {
        const std::string &nm = convs[c];
        int IC = 512, OC = 512;
        bool up = false;
        if (c > 0) {
            const int i = (int) c - 1, j = i / 2;
            up = (i % 2) == 0;
            IC = up ? ST_IC[j] : ST_OC[j];
            OC = ST_OC[j];
        }
        const std::vector<float> &W = d->t[nm];
        std::vector<float> &sa = d->saug[nm];
        sa.assign((size_t) (IC + 1) * OC, 0.0f);
        orc_saug(W.data(), IC, OC, sa.data());
        if (up) {
            const std::string kb = nm.substr(0, nm.size() - 6) + "blur.kernel";
            std::vector<float> &ts = d->tsub[nm];
            ts.assign((size_t) 4 * OC * 9 * IC, 0.0f);
            orc_tsubcf(W.data(), d->t[kb].data(), IC, OC, ts.data());
        }
    }
    d->prepared = true;
    return 0;
}

// the decoder graph, src/motion_dec.cpp:794-888 (mode 0) with the fast graph's
// sub-pixel up-conv as mode 1
int orc_dec_decode(orc_dec *d, const float *lat, int mode, int keep, float *img) {
    if (!d->prepared) {
        d->err = "decoder not prepared";
        return -1;
    }
    for (int j = 0; j < 7; j++)
        if (d->feat[j].empty()) {
            d->err = "feats not set";
            return -1;
        }
    d->taps.clear();
    // conv1 on the 4x4 constant input
    const int flags = mode & ~1;
    mode &= 1;
    std::vector<float> x = d->get("dec.input.input");
    x = styled_conv_exact(*d, x, 512, 4, "dec.conv1", lat, flags);
    d->tap(keep, "conv1_4", x.data(), x.size());
    std::vector<float> skip, skipf;  // rgb / flow accumulators, CHW [3][r][r]
    int IC = 512;
    for (int j = 0; j < 7; j++) {
        const int r = 8 << j, OC = ST_OC[j];
        const size_t N = (size_t) r * r;
        char b1[32], b2[32], bf[32], br[32];
        snprintf(b1, sizeof b1, "dec.convs.%d", 2 * j);
        snprintf(b2, sizeof b2, "dec.convs.%d", 2 * j + 1);
        snprintf(bf, sizeof bf, "dec.to_flows.%d", j);
        snprintf(br, sizeof br, "dec.to_rgbs.%d", j);
        const std::string R = "r" + std::to_string(r);

        std::vector<float> out = styled_conv_up(*d, x, IC, r / 2, b1, lat, mode, flags);
        d->tap(keep, R + ".conv1", out.data(), out.size());
        out = styled_conv_exact(*d, out, OC, r, b2, lat, flags);
        if (flags & ORC_F16_OUT) round16(out);
        d->tap(keep, R + ".conv2", out.data(), out.size());

        // ToFlow: 1x1 modulated conv (no demod) + bias + upsample2x(skip_flow)
        const std::vector<float> fs = d->style_of(std::string(bf) + ".conv", lat, (flags & ORC_F16_FOLD) != 0);
        const std::vector<float> &fW = d->get(std::string(bf) + ".conv.weight");
        const std::vector<float> &fb = d->get(std::string(bf) + ".bias");
        const std::vector<float> &fup = d->get(std::string(bf) + ".upsample.kernel");
        std::vector<float> fl((size_t) 3 * N);
#pragma omp parallel for schedule(static)
        for (size_t p = 0; p < N; p++)
            for (int k = 0; k < 3; k++) {
                float a = 0.0f;
                for (int c = 0; c < OC; c++)
                    a += fW[(size_t) k * OC + c] * (out[(size_t) c * N + p] * fs[(size_t) c]);
                fl[(size_t) k * N + p] = a + fb[(size_t) k];
            }
        if (!skipf.empty()) {
            std::vector<float> up((size_t) 3 * N);
            orc_upfirdn2x(skipf.data(), fup.data(), r / 2, r / 2, 3, up.data());
            for (size_t i = 0; i < fl.size(); i++) fl[i] += up[i];
        }
        skipf = fl;
        d->tap(keep, R + ".flowmap", fl.data(), fl.size());

        // grid (identity grid lin = -1 + 2i/(r-1), motion_dec.cpp:710-719)
        std::vector<double> lin((size_t) r);
        for (int i = 0; i < r; i++) lin[(size_t) i] = -1.0 + 2.0 * i / (r - 1);
        std::vector<float> grid((size_t) 2 * N), m(N);
        for (int yy = 0; yy < r; yy++)
            for (int xx = 0; xx < r; xx++) {
                const size_t p = (size_t) yy * r + xx;
                grid[2 * p + 0] = tanhf(fl[p]) + (float) lin[(size_t) xx];
                grid[2 * p + 1] = tanhf(fl[N + p]) + (float) lin[(size_t) yy];
                m[p] = 1.0f / (1.0f + expf(-fl[2 * N + p]));
            }
        d->tap(keep, R + ".grid", grid.data(), grid.size());

        std::vector<float> samp_cl((size_t) OC * N);
        std::vector<float> f16feat;
        if (flags & (ORC_F16_FEATS | ORC_F16_FOLD)) {
            f16feat = d->feat[j];
            round16(f16feat);
        }
        orc_bilinear_gather((flags & (ORC_F16_FEATS | ORC_F16_FOLD)) ? f16feat.data() : d->feat[j].data(), 0, OC, r,
                            r, grid.data(), (int64_t) N, 0, 0, samp_cl.data());
        std::vector<float> warp((size_t) OC * N), trunk((size_t) OC * N);
#pragma omp parallel for schedule(static)
        for (int c = 0; c < OC; c++)
            for (size_t p = 0; p < N; p++) {
                const float w = samp_cl[p * OC + c] * m[p];
                warp[(size_t) c * N + p] = w;
                trunk[(size_t) c * N + p] = w + out[(size_t) c * N + p] * (1.0f - m[p]);
            }
        d->tap(keep, R + ".warp", warp.data(), warp.size());
        d->tap(keep, R + ".out", trunk.data(), trunk.size());

        // ToRGB: 1x1 EqualConv + FusedLeakyReLU + bias + upsample2x(skip)
        const std::vector<float> &rW = d->get(std::string(br) + ".conv.0.weight");
        const std::vector<float> &rlb = d->get(std::string(br) + ".conv.1.bias");
        const std::vector<float> &rb = d->get(std::string(br) + ".bias");
        const std::vector<float> &rup = d->get(std::string(br) + ".upsample.kernel");
        std::vector<float> rgb((size_t) 3 * N);
#pragma omp parallel for schedule(static)
        for (size_t p = 0; p < N; p++)
            for (int k = 0; k < 3; k++) {
                float a = 0.0f;
                for (int c = 0; c < OC; c++) a += rW[(size_t) k * OC + c] * warp[(size_t) c * N + p];
                rgb[(size_t) k * N + p] = lrelu(a + rlb[(size_t) k], 0.2f) + rb[(size_t) k];
            }
        if (!skip.empty()) {
            std::vector<float> up((size_t) 3 * N);
            orc_upfirdn2x(skip.data(), rup.data(), r / 2, r / 2, 3, up.data());
            for (size_t i = 0; i < rgb.size(); i++) rgb[i] += up[i];
        }
        skip = rgb;
        d->tap(keep, R + ".rgb", rgb.data(), rgb.size());

        x.swap(trunk);
        IC = OC;
    }
    if (img) memcpy(img, skip.data(), skip.size() * 4);
    return 0;
}

int64_t orc_dec_tap(const orc_dec *d, const char *name, float *out, int64_t cap) {
    auto it = d->taps.find(name);
    if (it == d->taps.end()) return -1;
    const int64_t n = (int64_t) it->second.size();
    if (out && cap >= n) memcpy(out, it->second.data(), (size_t) n * 4);
    return n;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// motion encoder (src/motion_enc.cpp:46-184, ops src/ops_common.h:12-43)
// ---------------------------------------------------------------------------
namespace {

const int ENC_IN[7] = {32, 64, 128, 256, 512, 512, 512};    // motion_enc.cpp:46
const int ENC_OUT[7] = {64, 128, 256, 512, 512, 512, 512};  // motion_enc.cpp:47

std::map<std::string, int64_t> encoder_tensors() {
    std::map<std::string, int64_t> m;
    char nm[64];
    m["enc.net_app.convs.0.0.weight"] = 32 * 3;
    m["enc.net_app.convs.0.1.bias"] = 32;
    for (int i = 1; i <= 7; i++) {
        const int64_t C = ENC_IN[i - 1], Co = ENC_OUT[i - 1];
        auto put = [&](const char *suffix, int64_t n) {
            snprintf(nm, sizeof nm, "enc.net_app.convs.%d.%s", i, suffix);
            m[nm] = n;
        };
        put("conv1.0.weight", C * C * 9);
        put("conv1.1.bias", C);
        put("conv2.0.kernel", 16);
        put("conv2.1.weight", Co * C * 9);
        put("conv2.2.bias", Co);
        put("skip.0.kernel", 16);
        put("skip.1.weight", Co * C);
    }
    m["enc.net_app.convs.8.weight"] = (int64_t) 512 * 512 * 16;
    for (int i = 0; i < 5; i++) {
        const int64_t out = i == 4 ? 20 : 512;
        snprintf(nm, sizeof nm, "enc.fc.%d.weight", i);
        m[nm] = out * 512;
        snprintf(nm, sizeof nm, "enc.fc.%d.bias", i);
        m[nm] = out;
    }
    m["dec.direction.Q"] = 512 * 20;
    return m;
}

// y[OC][OH][OW] = corr2d(x[IC][IH][IW], w[OC][IC][K][K]) with stride s and
// zero padding p on every side (ggml_im2col + mul_mat, src/ops_common.h:12-26)
void conv2d_s(const float *x, int IC, int IH, int IW, const float *w, int OC, int K, int s,
              int p, int OH, int OW, float *y) {
    if (s == 1) {
        conv2d(x, IC, IH, IW, w, OC, K, K, p, p, OH, OW, y);
        return;
    }
#pragma omp parallel for collapse(2) schedule(dynamic, 4)
    for (int o = 0; o < OC; o++)
        for (int oy = 0; oy < OH; oy++) {
            float *out = y + ((size_t) o * OH + oy) * OW;
            for (int ox = 0; ox < OW; ox++) out[ox] = 0.0f;
            for (int ic = 0; ic < IC; ic++)
                for (int ky = 0; ky < K; ky++) {
                    const int iy = oy * s + ky - p;
                    if (iy < 0 || iy >= IH) continue;
                    const float *row = x + ((size_t) ic * IH + iy) * IW;
                    for (int kx = 0; kx < K; kx++) {
                        const float wv = w[(((size_t) o * IC + ic) * K + ky) * K + kx];
                        for (int ox = 0; ox < OW; ox++) {
                            const int ix = ox * s + kx - p;
                            if (ix >= 0 && ix < IW) out[ox] += wv * row[ix];
                        }
                    }
                }
        }
}

// FusedLeakyReLU with its sqrt2 folded upstream: lrelu(x + b), slope 0.2
void bias_lrelu_chw(std::vector<float> &x, const std::vector<float> &b, size_t P) {
    const int C = (int) b.size();
#pragma omp parallel for schedule(static)
    for (int c = 0; c < C; c++)
        for (size_t q = 0; q < P; q++) x[c * P + q] = lrelu(x[c * P + q] + b[(size_t) c], 0.2f);
}

}  // namespace

struct orc_enc {
    std::map<std::string, int64_t> spec = encoder_tensors();
    std::map<std::string, std::vector<float>> t;
    std::string err;
    const std::vector<float> &get(const std::string &n) const { return t.at(n); }
};

extern "C" {

orc_enc *orc_enc_create(void) { return new orc_enc(); }
void orc_enc_destroy(orc_enc *e) { delete e; }
const char *orc_enc_error(const orc_enc *e) { return e ? e->err.c_str() : "null encoder"; }

int orc_enc_set(orc_enc *e, const char *name, const float *data, int64_t n) {
    auto it = e->spec.find(name);
    if (it == e->spec.end() || it->second != n) {
        e->err = std::string("orc_enc_set: unknown tensor or size mismatch: ") + name;
        return -1;
    }
    e->t[name].assign(data, data + n);
    return 0;
}

int orc_enc_run(orc_enc *e, const float *image, float *appearance, float *lambda, float *motion,
                float *const feats[7]) {
    for (auto &kv : e->spec)
        if (!e->t.count(kv.first)) {
            e->err = "orc_enc_run: missing tensor " + kv.first;
            return -1;
        }
    // stem: 1x1 conv 3 -> 32 + FLReLU at 512x512
    int H = 512;
    std::vector<float> x((size_t) 32 * H * H);
    conv2d_s(image, 3, H, H, e->get("enc.net_app.convs.0.0.weight").data(), 32, 1, 1, 0, H, H,
             x.data());
    bias_lrelu_chw(x, e->get("enc.net_app.convs.0.1.bias"), (size_t) H * H);
    std::vector<std::vector<float>> pyr;
    pyr.push_back(x);
    char nm[96];
    for (int i = 1; i <= 7; i++) {
        const int C = ENC_IN[i - 1], Co = ENC_OUT[i - 1];
        auto T = [&](const char *suffix) -> const std::vector<float> & {
            snprintf(nm, sizeof nm, "enc.net_app.convs.%d.%s", i, suffix);
            return e->get(nm);
        };
        const size_t P = (size_t) H * H;
        const int h = H / 2;
        // main: conv1 (3x3, pad 1) + FLReLU, Blur pad (2,2), conv2 (3x3 s2) + FLReLU
        std::vector<float> x1((size_t) C * P);
        conv2d_s(x.data(), C, H, H, T("conv1.0.weight").data(), C, 3, 1, 1, H, H, x1.data());
        bias_lrelu_chw(x1, T("conv1.1.bias"), P);
        const int Hb = H + 1;  // H + 2 + 2 - 3
        std::vector<float> xb((size_t) C * Hb * Hb);
        orc_blur(x1.data(), T("conv2.0.kernel").data(), H, H, C, 2, 2, xb.data());
        std::vector<float> x2((size_t) Co * h * h);
        conv2d_s(xb.data(), C, Hb, Hb, T("conv2.1.weight").data(), Co, 3, 2, 0, h, h, x2.data());
        bias_lrelu_chw(x2, T("conv2.2.bias"), (size_t) h * h);
        // skip: Blur pad (1,1), 1x1 stride-2 conv (1/sqrt2 folded into it)
        const int Hs = H - 1;  // H + 1 + 1 - 3
        std::vector<float> sb((size_t) C * Hs * Hs);
        orc_blur(x.data(), T("skip.0.kernel").data(), H, H, C, 1, 1, sb.data());
        std::vector<float> sk((size_t) Co * h * h);
        conv2d_s(sb.data(), C, Hs, Hs, T("skip.1.weight").data(), Co, 1, 2, 0, h, h, sk.data());
        for (size_t q = 0; q < x2.size(); q++) x2[q] += sk[q];
        x.swap(x2);
        H = h;
        pyr.push_back(x);
    }
    // 4x4 valid conv on the 4x4 map -> appearance [512]
    std::vector<float> app(512);
    conv2d_s(x.data(), 512, 4, 4, e->get("enc.net_app.convs.8.weight").data(), 512, 4, 1, 0, 1, 1,
             app.data());
    // five plain EqualLinears (scale folded): h = W h + b
    std::vector<float> hcur = app;
    for (int i = 0; i < 5; i++) {
        snprintf(nm, sizeof nm, "enc.fc.%d.weight", i);
        const std::vector<float> &W = e->get(nm);
        snprintf(nm, sizeof nm, "enc.fc.%d.bias", i);
        const std::vector<float> &b = e->get(nm);
        const int out = (int) b.size();
        std::vector<float> nh((size_t) out);
        for (int o = 0; o < out; o++) {
            float a = 0.0f;
            for (int k = 0; k < 512; k++) a += W[(size_t) o * 512 + k] * hcur[(size_t) k];
            nh[(size_t) o] = a + b[(size_t) o];
        }
        hcur.swap(nh);
    }
    // motion = Q lambda, Q [512][20]
    const std::vector<float> &Q = e->get("dec.direction.Q");
    if (appearance) memcpy(appearance, app.data(), 512 * 4);
    if (lambda) memcpy(lambda, hcur.data(), 20 * 4);
    if (motion)
        for (int r = 0; r < 512; r++) {
            float a = 0.0f;
            for (int k = 0; k < 20; k++) a += Q[(size_t) r * 20 + k] * hcur[(size_t) k];
            motion[r] = a;
        }
    // feats[j] = conv{6-j}, channel-last [r*r][C]
    for (int j = 0; j < 7; j++) {
        if (!feats || !feats[j]) continue;
        const std::vector<float> &f = pyr[(size_t) (6 - j)];
        const int r = 8 << j, Cj = (int) (f.size() / ((size_t) r * r));
        for (int c = 0; c < Cj; c++)
            for (int q = 0; q < r * r; q++) feats[j][(size_t) q * Cj + c] = f[(size_t) c * r * r + q];
    }
    return 0;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// flow-matching transformer (src/fmt.cpp:9-211) and chunk sampler
// (src/pipeline.cpp:15-91)
// ---------------------------------------------------------------------------
namespace {

// y[m][n] = sum_k x[m][k] W[n][k] + b[n]  (torch Linear, W [N][K])
void linear_rows(const float *x, int M, int K, const float *W, const float *b, int N, float *y) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int m = 0; m < M; m++)
        for (int n = 0; n < N; n++) {
            const float *xr = x + (size_t) m * K, *wr = W + (size_t) n * K;
            float a = 0.0f;
            for (int k = 0; k < K; k++) a += xr[k] * wr[k];
            y[(size_t) m * N + n] = a + (b ? b[n] : 0.0f);
        }
}
inline float silu(float v) { return v / (1.0f + expf(-v)); }
inline float gelu_tanh(float v) {
    const float c = 0.7978845608028654f;  // sqrt(2/pi)
    return 0.5f * v * (1.0f + tanhf(c * (v + 0.044715f * v * v * v)));
}
// ggml_norm (no affine) then the adaLN modulation h*scale + h + shift
void norm_modulate(const float *x, int M, int H, float eps, const float *mod, int mod_stride,
                   int shift_off, int scale_off, float *y) {
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; m++) {
        const float *r = x + (size_t) m * H;
        double mean = 0;
        for (int i = 0; i < H; i++) mean += r[i];
        mean /= H;
        double var = 0;
        for (int i = 0; i < H; i++) var += (r[i] - mean) * (r[i] - mean);
        var /= H;
        const float inv = (float) (1.0 / sqrt(var + eps));
        const float *md = mod + (size_t) m * mod_stride;
        for (int i = 0; i < H; i++) {
            const float h = (float) (r[i] - mean) * inv;
            y[(size_t) m * H + i] = h * md[scale_off + i] + h + md[shift_off + i];
        }
    }
}

}  // namespace

struct orc_fmt {
    orc_fmt_config c{};
    int T = 0, CD = 0, FF = 0;
    std::map<std::string, int64_t> spec;
    std::map<std::string, std::vector<float>> t;
    std::string err;
    const std::vector<float> &get(const std::string &n) const { return t.at(n); }
};

extern "C" {

orc_fmt *orc_fmt_create(const orc_fmt_config *cfg) {
    orc_fmt *f = new orc_fmt();
    f->c = *cfg;
    const int H = cfg->dim_h;
    f->T = cfg->chunk_frames + cfg->prev_frames;
    f->CD = cfg->dim_w + cfg->dim_a + cfg->dim_e;
    f->FF = (int) (H * cfg->mlp_ratio);
    auto lin = [&](const std::string &n, int64_t out, int64_t in) {
        f->spec[n + ".weight"] = out * in;
        f->spec[n + ".bias"] = out;
    };
    lin("t_embedder.mlp.0", H, cfg->t_freq_dim);
    lin("t_embedder.mlp.2", H, H);
    lin("c_embedder", H, f->CD);
    lin("x_embedder.proj", H, cfg->dim_w);
    f->spec["pos_embed"] = (int64_t) f->T * H;
    for (int i = 0; i < cfg->depth; i++) {
        const std::string b = "blocks." + std::to_string(i) + ".";
        lin(b + "adaLN_modulation.1", 6 * H, H);
        lin(b + "attn.qkv", 3 * H, H);
        lin(b + "attn.proj", H, H);
        lin(b + "mlp.fc1", f->FF, H);
        lin(b + "mlp.fc2", H, f->FF);
    }
    lin("decoder.adaLN_modulation.1", 2 * H, H);
    lin("decoder.linear", cfg->dim_w, H);
    return f;
}
void orc_fmt_destroy(orc_fmt *f) { delete f; }
const char *orc_fmt_error(const orc_fmt *f) { return f ? f->err.c_str() : "null fmt"; }

int orc_fmt_set(orc_fmt *f, const char *name, const float *data, int64_t n) {
    auto it = f->spec.find(name);
    if (it == f->spec.end() || it->second != n) {
        f->err = std::string("orc_fmt_set: unknown tensor or size mismatch: ") + name;
        return -1;
    }
    f->t[name].assign(data, data + n);
    return 0;
}

int orc_fmt_forward(orc_fmt *f, const float *x60, const float *cond, float tt, float *v) {
    for (auto &kv : f->spec)
        if (!f->t.count(kv.first)) {
            f->err = "orc_fmt_forward: missing tensor " + kv.first;
            return -1;
        }
    const orc_fmt_config &c = f->c;
    const int H = c.dim_h, T = f->T, B = 3, M = B * T, nh = c.n_heads, hd = H / nh;
    // timestep embedding: GLIDE sinusoid, freq_k = exp(-ln(10000) k / half)
    const int half = c.t_freq_dim / 2;
    std::vector<float> tf((size_t) c.t_freq_dim);
    for (int k = 0; k < half; k++) {
        const float fr = (float) exp(-log(10000.0) * (double) k / (double) half);
        tf[(size_t) k] = cosf(tt * fr);
        tf[(size_t) (half + k)] = sinf(tt * fr);
    }
    std::vector<float> te0((size_t) H), te((size_t) H);
    linear_rows(tf.data(), 1, c.t_freq_dim, f->get("t_embedder.mlp.0.weight").data(),
                f->get("t_embedder.mlp.0.bias").data(), H, te0.data());
    for (float &q : te0) q = silu(q);
    linear_rows(te0.data(), 1, H, f->get("t_embedder.mlp.2.weight").data(),
                f->get("t_embedder.mlp.2.bias").data(), H, te.data());
    // conditioning: silu(c_embedder(cond) + t_emb) per (branch, frame)
    std::vector<float> sc((size_t) M * H);
    linear_rows(cond, M, f->CD, f->get("c_embedder.weight").data(), f->get("c_embedder.bias").data(), H,
                sc.data());
    for (int m = 0; m < M; m++)
        for (int i = 0; i < H; i++) sc[(size_t) m * H + i] = silu(sc[(size_t) m * H + i] + te[(size_t) i]);
    // tokens: x_embedder(x60) + pos, the same rows in every branch
    std::vector<float> x1((size_t) T * H), x((size_t) M * H);
    linear_rows(x60, T, c.dim_w, f->get("x_embedder.proj.weight").data(),
                f->get("x_embedder.proj.bias").data(), H, x1.data());
    const std::vector<float> &pos = f->get("pos_embed");
    for (int b = 0; b < B; b++)
        for (int r = 0; r < T; r++)
            for (int i = 0; i < H; i++)
                x[((size_t) b * T + r) * H + i] = x1[(size_t) r * H + i] + pos[(size_t) r * H + i];
    std::vector<float> mod((size_t) M * 6 * H), h((size_t) M * H), qkv((size_t) M * 3 * H),
        att((size_t) M * H), o((size_t) M * H), m1((size_t) M * f->FF);
    const float scale = 1.0f / sqrtf((float) hd);
    for (int l = 0; l < c.depth; l++) {
        const std::string bn = "blocks." + std::to_string(l) + ".";
        auto W = [&](const std::string &n) { return f->get(bn + n + ".weight").data(); };
        auto Bv = [&](const std::string &n) { return f->get(bn + n + ".bias").data(); };
        linear_rows(sc.data(), M, H, W("adaLN_modulation.1"), Bv("adaLN_modulation.1"), 6 * H, mod.data());
        // attention branch (chunks: shift, scale, gate for msa then for mlp)
        norm_modulate(x.data(), M, H, c.ln_eps, mod.data(), 6 * H, 0, H, h.data());
        linear_rows(h.data(), M, H, W("attn.qkv"), Bv("attn.qkv"), 3 * H, qkv.data());
        // banded mask: row i attends cols [max(0,i-w), i+w+1), scale 1/sqrt(hd)
#pragma omp parallel for collapse(3) schedule(static)
        for (int b = 0; b < B; b++)
            for (int hh = 0; hh < nh; hh++)
                for (int i = 0; i < T; i++) {
                    const int j0 = std::max(0, i - c.attn_window), j1 = std::min(T, i + c.attn_window + 1);
                    const float *q = qkv.data() + ((size_t) b * T + i) * 3 * H + hh * hd;
                    float sc_[64];
                    float mx = -INFINITY;
                    for (int j = j0; j < j1; j++) {
                        const float *k = qkv.data() + ((size_t) b * T + j) * 3 * H + H + hh * hd;
                        float a = 0.0f;
                        for (int d = 0; d < hd; d++) a += q[d] * k[d];
                        sc_[j - j0] = a * scale;
                        mx = std::max(mx, sc_[j - j0]);
                    }
                    float sum = 0.0f;
                    for (int j = j0; j < j1; j++) sum += (sc_[j - j0] = expf(sc_[j - j0] - mx));
                    float *out = att.data() + ((size_t) b * T + i) * H + hh * hd;
                    for (int d = 0; d < hd; d++) out[d] = 0.0f;
                    for (int j = j0; j < j1; j++) {
                        const float pj = sc_[j - j0] / sum;
                        const float *vv = qkv.data() + ((size_t) b * T + j) * 3 * H + 2 * H + hh * hd;
                        for (int d = 0; d < hd; d++) out[d] += pj * vv[d];
                    }
                }
        linear_rows(att.data(), M, H, W("attn.proj"), Bv("attn.proj"), H, o.data());
        for (int m = 0; m < M; m++)
            for (int i = 0; i < H; i++)
                x[(size_t) m * H + i] += mod[(size_t) m * 6 * H + 2 * H + i] * o[(size_t) m * H + i];
        // MLP branch (tanh GELU)
        norm_modulate(x.data(), M, H, c.ln_eps, mod.data(), 6 * H, 3 * H, 4 * H, h.data());
        linear_rows(h.data(), M, H, W("mlp.fc1"), Bv("mlp.fc1"), f->FF, m1.data());
        for (float &q : m1) q = gelu_tanh(q);
        linear_rows(m1.data(), M, f->FF, W("mlp.fc2"), Bv("mlp.fc2"), H, o.data());
        for (int m = 0; m < M; m++)
            for (int i = 0; i < H; i++)
                x[(size_t) m * H + i] += mod[(size_t) m * 6 * H + 5 * H + i] * o[(size_t) m * H + i];
    }
    std::vector<float> fm((size_t) M * 2 * H);
    linear_rows(sc.data(), M, H, f->get("decoder.adaLN_modulation.1.weight").data(),
                f->get("decoder.adaLN_modulation.1.bias").data(), 2 * H, fm.data());
    norm_modulate(x.data(), M, H, c.ln_eps, fm.data(), 2 * H, 0, H, h.data());
    linear_rows(h.data(), M, H, f->get("decoder.linear.weight").data(), f->get("decoder.linear.bias").data(),
                c.dim_w, v);
    return 0;
}

int orc_fmt_sample(orc_fmt *f, const float *wr, const float *prev_wa, const float *cond_audio,
                   const float *prev_x, const float *x0, int emotion, float *motion) {
    const orc_fmt_config &c = f->c;
    const int T = f->T, P = c.prev_frames, CF = c.chunk_frames, D = c.dim_w, CD = f->CD;
    // condition rows [wr | wa | we] per branch: uncond nulls the current
    // frames' wa and we, audio-only nulls we; prev_wa rows stay in all
    std::vector<float> cond((size_t) 3 * T * CD, 0.0f);
    for (int b = 0; b < 3; b++)
        for (int fr = 0; fr < T; fr++) {
            float *row = cond.data() + ((size_t) b * T + fr) * CD;
            memcpy(row, wr, (size_t) D * 4);
            const float *wa = fr < P ? prev_wa + (size_t) fr * D : cond_audio + (size_t) (fr - P) * D;
            if (!(b == 0 && fr >= P)) memcpy(row + D, wa, (size_t) D * 4);
            if (b == 1 && emotion >= 0 && emotion < c.dim_e) row[D + c.dim_a + emotion] = 1.0f;
        }
    std::vector<float> x((size_t) CF * D), x60((size_t) T * D), v((size_t) 3 * T * D);
    memcpy(x.data(), x0, x.size() * 4);
    memcpy(x60.data(), prev_x, (size_t) P * D * 4);
    for (int s = 0; s < c.nfe - 1; s++) {
        memcpy(x60.data() + (size_t) P * D, x.data(), x.size() * 4);
        const float t0 = (float) ((double) s / (double) (c.nfe - 1));
        const float t1 = (float) ((double) (s + 1) / (double) (c.nfe - 1));
        if (orc_fmt_forward(f, x60.data(), cond.data(), t0, v.data()) != 0) return -1;
        const float *u = v.data(), *fu = v.data() + (size_t) T * D, *a = v.data() + (size_t) 2 * T * D;
        const float dt = t1 - t0;
        for (int fr = 0; fr < CF; fr++)
            for (int i = 0; i < D; i++) {
                const size_t q = (size_t) (P + fr) * D + i;
                const float vc = (u[q] + c.a_cfg * (a[q] - u[q])) + c.e_cfg * (fu[q] - a[q]);
                x[(size_t) fr * D + i] = x[(size_t) fr * D + i] + dt * vc;
            }
    }
    memcpy(motion, x.data(), x.size() * 4);
    return 0;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// audio encoder (src/audio_enc.cpp:55-236)
// ---------------------------------------------------------------------------
namespace {

inline float gelu_erf(float v) { return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f)); }

// per row of [M][N]: (x - mean)/sqrt(var + eps) * w + b (ggml_norm then affine)
void layer_norm_rows(float *x, int64_t M, int N, const float *w, const float *b, float eps) {
#pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; m++) {
        float *r = x + m * N;
        double mean = 0;
        for (int i = 0; i < N; i++) mean += r[i];
        mean /= N;
        double var = 0;
        for (int i = 0; i < N; i++) var += (r[i] - mean) * (r[i] - mean);
        var /= N;
        const float inv = (float) (1.0 / sqrt(var + eps));
        for (int i = 0; i < N; i++) r[i] = (float) (r[i] - mean) * inv * (w ? w[i] : 1.0f) + (b ? b[i] : 0.0f);
    }
}

// y[t][o] = sum_{k,c} W[o][c][k] x[t*s + k - p][c] (zero outside), x [T][C]
// time-major channel-last, W torch [O][C][K]
void conv1d_tc(const float *x, int64_t T, int C, const float *W, int O, int K, int s, int p, int64_t OT,
               float *y) {
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < OT; t++)
        for (int o = 0; o < O; o++) {
            float a = 0.0f;
            for (int k = 0; k < K; k++) {
                const int64_t ti = t * s + k - p;
                if (ti < 0 || ti >= T) continue;
                const float *xr = x + ti * C;
                const float *wr = W + (size_t) o * C * K + k;
                for (int c = 0; c < C; c++) a += wr[(size_t) c * K] * xr[c];
            }
            y[t * O + o] = a;
        }
}

}  // namespace

struct orc_aud {
    orc_aud_config c{};
    std::map<std::string, int64_t> spec;
    std::map<std::string, std::vector<float>> t;
    std::string err;
    const std::vector<float> &get(const std::string &n) const { return t.at(n); }
};

extern "C" {

orc_aud *orc_aud_create(const orc_aud_config *cfg) {
    orc_aud *a = new orc_aud();
    a->c = *cfg;
    const int Hd = cfg->hidden, F = cfg->ffn;
    int ic = 1;
    for (int i = 0; i < 7; i++) {
        a->spec["feature_extractor.conv_layers." + std::to_string(i) + ".conv.weight"] =
            (int64_t) cfg->conv_dim[i] * ic * cfg->conv_kernel[i];
        ic = cfg->conv_dim[i];
    }
    a->spec["feature_extractor.conv_layers.0.layer_norm.weight"] = cfg->conv_dim[0];
    a->spec["feature_extractor.conv_layers.0.layer_norm.bias"] = cfg->conv_dim[0];
    const int C = cfg->conv_dim[6];
    a->spec["feature_projection.layer_norm.weight"] = C;
    a->spec["feature_projection.layer_norm.bias"] = C;
    a->spec["feature_projection.projection.weight"] = (int64_t) Hd * C;
    a->spec["feature_projection.projection.bias"] = Hd;
    a->spec["encoder.pos_conv_embed.conv.weight"] = (int64_t) Hd * (Hd / cfg->pos_groups) * cfg->pos_kernel;
    a->spec["encoder.pos_conv_embed.conv.bias"] = Hd;
    a->spec["encoder.layer_norm.weight"] = Hd;
    a->spec["encoder.layer_norm.bias"] = Hd;
    for (int i = 0; i < cfg->n_layers; i++) {
        const std::string b = "encoder.layers." + std::to_string(i) + ".";
        for (const char *pj : {"q_proj", "k_proj", "v_proj", "out_proj"}) {
            a->spec[b + "attention." + pj + ".weight"] = (int64_t) Hd * Hd;
            a->spec[b + "attention." + pj + ".bias"] = Hd;
        }
        a->spec[b + "layer_norm.weight"] = Hd;
        a->spec[b + "layer_norm.bias"] = Hd;
        a->spec[b + "feed_forward.intermediate_dense.weight"] = (int64_t) F * Hd;
        a->spec[b + "feed_forward.intermediate_dense.bias"] = F;
        a->spec[b + "feed_forward.output_dense.weight"] = (int64_t) Hd * F;
        a->spec[b + "feed_forward.output_dense.bias"] = Hd;
        a->spec[b + "final_layer_norm.weight"] = Hd;
        a->spec[b + "final_layer_norm.bias"] = Hd;
    }
    a->spec["audio_projection.0.weight"] = (int64_t) cfg->dim_w * Hd * cfg->n_layers;
    a->spec["audio_projection.0.bias"] = cfg->dim_w;
    a->spec["audio_projection.1.weight"] = cfg->dim_w;
    a->spec["audio_projection.1.bias"] = cfg->dim_w;
    return a;
}
void orc_aud_destroy(orc_aud *a) { delete a; }
const char *orc_aud_error(const orc_aud *a) { return a ? a->err.c_str() : "null audio encoder"; }

int orc_aud_set(orc_aud *a, const char *name, const float *data, int64_t n) {
    auto it = a->spec.find(name);
    if (it == a->spec.end() || it->second != n) {
        a->err = std::string("orc_aud_set: unknown tensor or size mismatch: ") + name;
        return -1;
    }
    a->t[name].assign(data, data + n);
    return 0;
}

int orc_aud_encode(orc_aud *a, const float *audio, int64_t n_in, int64_t seq_len, float *wa) {
    for (auto &kv : a->spec)
        if (!a->t.count(kv.first)) {
            a->err = "orc_aud_encode: missing tensor " + kv.first;
            return -1;
        }
    const orc_aud_config &c = a->c;
    // replicate-pad (or crop) to exactly seq_len * sample_rate / fps samples
    // unless already a multiple of it (src/audio_enc.cpp:60-70)
    const int64_t unit = (int64_t) (seq_len * c.sample_rate / c.fps);
    int64_t n = n_in;
    std::vector<float> x;
    if (unit > 0 && n % unit != 0) {
        n = unit;
        x.assign((size_t) n, n_in > 0 ? audio[n_in - 1] : 0.0f);
        memcpy(x.data(), audio, (size_t) std::min(n, n_in) * 4);
    } else {
        x.assign(audio, audio + n);
    }
    // conv stack, time-major [T][C]
    int64_t T = n;
    int C = 1;
    for (int i = 0; i < 7; i++) {
        const int K = c.conv_kernel[i], s = c.conv_stride[i], O = c.conv_dim[i];
        const int64_t OT = (T - K) / s + 1;
        if (OT < 1) {
            a->err = "audio too short";
            return -1;
        }
        std::vector<float> y((size_t) OT * O);
        conv1d_tc(x.data(), T, C, a->get("feature_extractor.conv_layers." + std::to_string(i) + ".conv.weight").data(),
                  O, K, s, 0, OT, y.data());
        if (i == 0) {
            // GroupNorm with one group per channel: norm over time + affine
            const std::vector<float> &gw = a->get("feature_extractor.conv_layers.0.layer_norm.weight");
            const std::vector<float> &gb = a->get("feature_extractor.conv_layers.0.layer_norm.bias");
#pragma omp parallel for schedule(static)
            for (int o = 0; o < O; o++) {
                double mean = 0;
                for (int64_t t = 0; t < OT; t++) mean += y[(size_t) t * O + o];
                mean /= (double) OT;
                double var = 0;
                for (int64_t t = 0; t < OT; t++) {
                    const double d = y[(size_t) t * O + o] - mean;
                    var += d * d;
                }
                var /= (double) OT;
                const float inv = (float) (1.0 / sqrt(var + c.ln_eps));
                for (int64_t t = 0; t < OT; t++)
                    y[(size_t) t * O + o] = (float) (y[(size_t) t * O + o] - mean) * inv * gw[(size_t) o] + gb[(size_t) o];
            }
        }
        for (float &v : y) v = gelu_erf(v);
        x.swap(y);
        T = OT;
        C = O;
    }
    if (T < 2 || seq_len < 1) {
        a->err = "audio too short";
        return -1;
    }
    // linear interpolation, align_corners=True, to seq_len frames
    const int64_t S = seq_len;
    std::vector<float> h((size_t) S * C, 0.0f);
    for (int64_t s = 0; s < S; s++) {
        const double pos = S == 1 ? 0.0 : (double) s * (double) (T - 1) / (double) (S - 1);
        int64_t i0 = (int64_t) pos;
        if (i0 > T - 1) i0 = T - 1;
        const double frac = pos - (double) i0;
        const float w0 = (float) (1.0 - frac), w1 = (float) frac;
        for (int ch = 0; ch < C; ch++) {
            float v = w0 * x[(size_t) i0 * C + ch];
            if (i0 + 1 < T && frac > 0) v += w1 * x[(size_t) (i0 + 1) * C + ch];
            h[(size_t) s * C + ch] = v;
        }
    }
    // feature projection: LayerNorm + Linear(C -> hidden)
    const int Hd = c.hidden;
    layer_norm_rows(h.data(), S, C, a->get("feature_projection.layer_norm.weight").data(),
                    a->get("feature_projection.layer_norm.bias").data(), c.ln_eps);
    std::vector<float> e((size_t) S * Hd);
    linear_rows(h.data(), (int) S, C, a->get("feature_projection.projection.weight").data(),
                a->get("feature_projection.projection.bias").data(), Hd, e.data());
    // positional conv: grouped conv1d (K taps, pad K/2), drop the last step, GELU, add
    {
        const int G = c.pos_groups, cg = Hd / G, K = c.pos_kernel, pad = K / 2;
        const std::vector<float> &pw = a->get("encoder.pos_conv_embed.conv.weight");
        const std::vector<float> &pb = a->get("encoder.pos_conv_embed.conv.bias");
        std::vector<float> pos((size_t) S * Hd);
#pragma omp parallel for collapse(2) schedule(static)
        for (int64_t t = 0; t < S; t++)
            for (int o = 0; o < Hd; o++) {
                const int g = o / cg;
                float acc = 0.0f;
                for (int k = 0; k < K; k++) {
                    const int64_t ti = t + k - pad;
                    if (ti < 0 || ti >= S) continue;
                    const float *xr = e.data() + (size_t) ti * Hd + (size_t) g * cg;
                    const float *wr = pw.data() + ((size_t) o * cg) * K + k;
                    for (int ci = 0; ci < cg; ci++) acc += wr[(size_t) ci * K] * xr[ci];
                }
                pos[(size_t) t * Hd + o] = gelu_erf(acc + pb[(size_t) o]);
            }
        for (size_t q = 0; q < e.size(); q++) e[q] += pos[q];
    }
    layer_norm_rows(e.data(), S, Hd, a->get("encoder.layer_norm.weight").data(),
                    a->get("encoder.layer_norm.bias").data(), c.ln_eps);
    // post-norm transformer; all layer outputs stacked per frame
    const int nh = c.n_heads, hd = Hd / nh, F = c.ffn, L = c.n_layers;
    const float scaling = 1.0f / sqrtf((float) hd);
    std::vector<float> stacked((size_t) S * Hd * L), q((size_t) S * Hd), k((size_t) S * Hd),
        v((size_t) S * Hd), att((size_t) S * Hd), o((size_t) S * Hd), f1((size_t) S * F);
    for (int l = 0; l < L; l++) {
        const std::string b = "encoder.layers." + std::to_string(l) + ".";
        auto W = [&](const std::string &n) { return a->get(b + n + ".weight").data(); };
        auto B = [&](const std::string &n) { return a->get(b + n + ".bias").data(); };
        linear_rows(e.data(), (int) S, Hd, W("attention.q_proj"), B("attention.q_proj"), Hd, q.data());
        for (float &z : q) z *= scaling;
        linear_rows(e.data(), (int) S, Hd, W("attention.k_proj"), B("attention.k_proj"), Hd, k.data());
        linear_rows(e.data(), (int) S, Hd, W("attention.v_proj"), B("attention.v_proj"), Hd, v.data());
#pragma omp parallel
        {
            std::vector<float> sc((size_t) S);
#pragma omp for collapse(2) schedule(static)
            for (int hh = 0; hh < nh; hh++)
                for (int64_t i = 0; i < S; i++) {
                    const float *qi = q.data() + (size_t) i * Hd + hh * hd;
                    float mx = -INFINITY;
                    for (int64_t j = 0; j < S; j++) {
                        const float *kj = k.data() + (size_t) j * Hd + hh * hd;
                        float d = 0.0f;
                        for (int z = 0; z < hd; z++) d += qi[z] * kj[z];
                        sc[(size_t) j] = d;
                        mx = std::max(mx, d);
                    }
                    float sum = 0.0f;
                    for (int64_t j = 0; j < S; j++) sum += (sc[(size_t) j] = expf(sc[(size_t) j] - mx));
                    float *out = att.data() + (size_t) i * Hd + hh * hd;
                    for (int z = 0; z < hd; z++) out[z] = 0.0f;
                    for (int64_t j = 0; j < S; j++) {
                        const float pj = sc[(size_t) j] / sum;
                        const float *vj = v.data() + (size_t) j * Hd + hh * hd;
                        for (int z = 0; z < hd; z++) out[z] += pj * vj[z];
                    }
                }
        }
        linear_rows(att.data(), (int) S, Hd, W("attention.out_proj"), B("attention.out_proj"), Hd, o.data());
        for (size_t z = 0; z < e.size(); z++) e[z] += o[z];
        layer_norm_rows(e.data(), S, Hd, W("layer_norm"), B("layer_norm"), c.ln_eps);
        linear_rows(e.data(), (int) S, Hd, W("feed_forward.intermediate_dense"), B("feed_forward.intermediate_dense"),
                    F, f1.data());
        for (float &z : f1) z = gelu_erf(z);
        linear_rows(f1.data(), (int) S, F, W("feed_forward.output_dense"), B("feed_forward.output_dense"), Hd,
                    o.data());
        for (size_t z = 0; z < e.size(); z++) e[z] += o[z];
        layer_norm_rows(e.data(), S, Hd, W("final_layer_norm"), B("final_layer_norm"), c.ln_eps);
        for (int64_t s = 0; s < S; s++)
            memcpy(stacked.data() + ((size_t) s * L + l) * Hd, e.data() + (size_t) s * Hd, (size_t) Hd * 4);
    }
    // audio projection: Linear(L*hidden -> dim_w) + LayerNorm(eps 1e-5) + SiLU
    linear_rows(stacked.data(), (int) S, Hd * L, a->get("audio_projection.0.weight").data(),
                a->get("audio_projection.0.bias").data(), c.dim_w, wa);
    layer_norm_rows(wa, S, c.dim_w, a->get("audio_projection.1.weight").data(),
                    a->get("audio_projection.1.bias").data(), 1e-5f);
    for (int64_t z = 0; z < S * c.dim_w; z++) wa[z] = silu(wa[z]);
    return 0;
}

}  // extern "C"


// ---------------------------------------------------------------------------
// CHW f32 frame -> RGB24 bytes (tools/tp-cli.cpp:43-53, the frame the CLI
// hands to its video encoder): clamp with the same comparisons, then
// (unsigned char) ((v + 1) / 2 * 255) in f32, truncating toward zero
// ---------------------------------------------------------------------------
extern "C" void orc_chw_to_rgb24(const float *chw, int64_t n, int64_t hw, unsigned char *rgb) {
    for (int64_t f = 0; f < n; f++)
        for (int64_t i = 0; i < hw; i++)
            for (int c = 0; c < 3; c++) {
                float v = chw[(f * 3 + c) * hw + i];
                v = v < -1 ? -1 : (v > 1 ? 1 : v);
                rgb[(f * hw + i) * 3 + c] = (unsigned char) ((v + 1.0f) / 2.0f * 255.0f);
            }
}
