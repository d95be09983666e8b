// C entry points over the reference's own op code (appended by
// oracle/ref_build.py after the code it extracts from the patch, so the
// kernels and forward functions named here are the reference's, compiled as
// host code). TEST INFRASTRUCTURE ONLY.
//
// ref_cpu_*: the patched ggml CPU forward functions (patch:319-657), called
//            single-threaded (ith 0 of nth 1).
// ref_cu_*:  the patched CUDA kernels (patch:688-718, 830-861, 920-1095), run
//            by looping one host thread over every block and thread index.

thread_local ref_dim3 blockIdx, threadIdx, blockDim;

namespace {

void set_f32(ggml_tensor &t, void *data, int64_t n0, int64_t n1 = 1, int64_t n2 = 1,
             int64_t n3 = 1, ggml_type ty = GGML_TYPE_F32) {
    t.type = ty;
    t.ne[0] = n0;
    t.ne[1] = n1;
    t.ne[2] = n2;
    t.ne[3] = n3;
    const size_t es = ty == GGML_TYPE_F16 ? 2 : 4;
    t.nb[0] = es;
    t.nb[1] = es * n0;
    t.nb[2] = t.nb[1] * n1;
    t.nb[3] = t.nb[2] * n2;
    t.data = data;
}

// launch emulation for kernels that compute i = blockIdx.x*blockDim.x + threadIdx.x
template <typename F>
void run_flat(int64_t total, F &&body) {
    blockDim.x = 1;
    threadIdx.x = 0;
    for (int64_t i = 0; i < total; i++) {
        blockIdx.x = (unsigned) i;
        body();
    }
}

}  // namespace

extern "C" {

// ---- CPU forward functions -------------------------------------------------
void ref_cpu_bilinear_gather(const void *feat, int f16, int C, int W, int H,
                             const float *grid, int64_t N, int planar, int sp, float *dst) {
    ggml_tensor a, b, d;
    set_f32(a, (void *) feat, C, (int64_t) W * H, 1, 1, f16 ? GGML_TYPE_F16 : GGML_TYPE_F32);
    if (planar)
        set_f32(b, (void *) grid, N, 2);
    else
        set_f32(b, (void *) grid, 2, N);
    if (sp)
        set_f32(d, dst, N, C);
    else
        set_f32(d, dst, C, N);
    d.op_params[0] = W;
    d.op_params[1] = H;
    d.op_params[2] = sp;
    d.op_params[3] = planar;
    d.src[0] = &a;
    d.src[1] = &b;
    ggml_compute_params p;
    ggml_compute_forward_bilinear_gather(&p, &d);
}

void ref_cpu_bias_lrelu(const float *x, const float *bias, const int64_t *ne, int axis,
                        float slope, float *y) {
    ggml_tensor a, b, d;
    set_f32(a, (void *) x, ne[0], ne[1], ne[2], ne[3]);
    set_f32(b, (void *) bias, ne[axis]);
    set_f32(d, y, ne[0], ne[1], ne[2], ne[3]);
    d.op_params[0] = axis;
    memcpy(&d.op_params[1], &slope, 4);
    d.src[0] = &a;
    d.src[1] = &b;
    ggml_compute_params p;
    ggml_compute_forward_bias_lrelu(&p, &d);
}

void ref_cpu_subpix_lrelu(const float *g0, const float *g1, const float *bias, int W,
                          int H, int OC, float slope, float *y) {
    ggml_tensor a, b, c, d;
    set_f32(a, (void *) g0, W, H, 2 * OC);
    set_f32(b, (void *) g1, W, H, 2 * OC);
    set_f32(c, (void *) bias, OC);
    set_f32(d, y, 2 * W, 2 * H, OC);
    memcpy(&d.op_params[0], &slope, 4);
    d.src[0] = &a;
    d.src[1] = &b;
    d.src[2] = &c;
    ggml_compute_params p;
    ggml_compute_forward_subpix_lrelu(&p, &d);
}

void ref_cpu_subpix_lrelu_cl(const float *y4, const float *bias, int OC, int64_t N,
                             int64_t B, int W, float slope, float *y) {
    ggml_tensor a, b, d;
    set_f32(a, (void *) y4, 4 * OC, N, B);
    set_f32(b, (void *) bias, OC);
    set_f32(d, y, OC, 4 * N, B);
    d.op_params[0] = W;
    memcpy(&d.op_params[1], &slope, 4);
    d.src[0] = &a;
    d.src[1] = &b;
    ggml_compute_params p;
    ggml_compute_forward_subpix_lrelu_cl(&p, &d);
}

void ref_cpu_upfirdn2x(const float *x, const float *k4, int W, int H, int64_t CB, float *y) {
    ggml_tensor a, b, d;
    set_f32(a, (void *) x, W, H, CB);
    set_f32(b, (void *) k4, 4, 4);
    set_f32(d, y, 2 * W, 2 * H, CB);
    d.src[0] = &a;
    d.src[1] = &b;
    ggml_compute_params p;
    ggml_compute_forward_upfirdn2x(&p, &d);
}

void ref_cpu_clsp_mul(const float *cl, const float *m, int C, int64_t N, float *y) {
    ggml_tensor a, b, d;
    set_f32(a, (void *) cl, C, N);
    set_f32(b, (void *) m, N);
    set_f32(d, y, N, C);
    d.src[0] = &a;
    d.src[1] = &b;
    ggml_compute_params p;
    ggml_compute_forward_clsp_mul(&p, &d);
}

void ref_cpu_clsp_lerp(const float *cl, const float *m, const float *o, int C, int64_t N,
                       float *y) {
    ggml_tensor a, b, c, d;
    set_f32(a, (void *) cl, C, N);
    set_f32(b, (void *) m, N);
    set_f32(c, (void *) o, N, C);
    set_f32(d, y, N, C);
    d.src[0] = &a;
    d.src[1] = &b;
    d.src[2] = &c;
    ggml_compute_params p;
    ggml_compute_forward_clsp_lerp(&p, &d);
}

void ref_cpu_flow_grid(const float *fl, const float *xs, int64_t N, float *y) {
    ggml_tensor a, b, d;
    set_f32(a, (void *) fl, N, 1, 3);
    set_f32(b, (void *) xs, N, 2);
    set_f32(d, y, N, 3);
    d.src[0] = &a;
    d.src[1] = &b;
    ggml_compute_params p;
    ggml_compute_forward_flow_grid(&p, &d);
}

// ---- CUDA kernels run on the host ----------------------------------------
void ref_cu_bilinear_gather(const void *feat, int f16, int C, int W, int H,
                            const float *grid, int64_t N, int planar, int sp, float *dst) {
    const int64_t total = (int64_t) C * N;
    if (f16) {
        if (sp)
            run_flat(total, [&] {
                bilinear_gather_kernel<half, true>((const half *) feat, grid, dst, C, W, H, N,
                                                   total, planar != 0);
            });
        else
            run_flat(total, [&] {
                bilinear_gather_kernel<half, false>((const half *) feat, grid, dst, C, W, H, N,
                                                    total, planar != 0);
            });
    } else {
        if (sp)
            run_flat(total, [&] {
                bilinear_gather_kernel<float, true>((const float *) feat, grid, dst, C, W, H, N,
                                                    total, planar != 0);
            });
        else
            run_flat(total, [&] {
                bilinear_gather_kernel<float, false>((const float *) feat, grid, dst, C, W, H,
                                                     N, total, planar != 0);
            });
    }
}

void ref_cu_im2col_cf(const float *src, int IC, int IW, int IH, int N, int KW, int KH,
                      int s0, int s1, int p0, int p1, int d0, int d1, void *dst, int dst_f16) {
    const int OW = (IW + 2 * p0 - d0 * (KW - 1) - 1) / s0 + 1;
    const int OH = (IH + 2 * p1 - d1 * (KH - 1) - 1) / s1 + 1;
    const int R = IC * KW * KH;
    const bool pow2 = (IC & (IC - 1)) == 0;
    int ic_shift = 0;
    while ((1 << ic_shift) < IC) ic_shift++;
    blockDim.x = 1;
    threadIdx.x = 0;
    for (int n = 0; n < OW * OH * N; n++) {
        blockIdx.x = (unsigned) n;
        if (dst_f16) {
            if (pow2)
                im2col_cf_kernel<half, true>(src, (half *) dst, IC, ic_shift, IW, IH, OW, OH, R,
                                             s0, s1, p0, p1, d0, d1, KW);
            else
                im2col_cf_kernel<half, false>(src, (half *) dst, IC, ic_shift, IW, IH, OW, OH, R,
                                              s0, s1, p0, p1, d0, d1, KW);
        } else {
            if (pow2)
                im2col_cf_kernel<float, true>(src, (float *) dst, IC, ic_shift, IW, IH, OW, OH,
                                              R, s0, s1, p0, p1, d0, d1, KW);
            else
                im2col_cf_kernel<float, false>(src, (float *) dst, IC, ic_shift, IW, IH, OW, OH,
                                               R, s0, s1, p0, p1, d0, d1, KW);
        }
    }
}

void ref_cu_bias_lrelu(const float *x, const float *bias, const int64_t *ne, int axis,
                       float slope, float *y) {
    const int64_t n = ne[0] * ne[1] * ne[2] * ne[3];
    const int C = (int) ne[axis];
    const int64_t d01 = ne[0] * ne[1];
    run_flat(n, [&] { bias_lrelu_kernel(x, bias, y, n, C, d01, axis, slope); });
}

void ref_cu_subpix_lrelu(const float *g0, const float *g1, const float *bias, int W, int H,
                         int OC, float slope, float *y) {
    const int64_t n = (int64_t) 4 * W * H * OC;
    run_flat(n, [&] { subpix_lrelu_kernel(g0, g1, bias, y, n, W, H, OC, slope); });
}

void ref_cu_subpix_lrelu_cl(const float *y4, const float *bias, int OC, int64_t N, int64_t B,
                            int W, float slope, float *y) {
    const int64_t n = (int64_t) OC * 4 * N * B;
    run_flat(n, [&] { subpix_lrelu_cl_kernel(y4, bias, y, n, OC, N, W, slope); });
}

void ref_cu_upfirdn2x(const float *x, const float *k4, int W, int H, int64_t CB, float *y) {
    const int64_t n = (int64_t) 4 * W * H * CB;
    run_flat(n, [&] { upfirdn2x_kernel(x, k4, y, n, W, H); });
}

void ref_cu_clsp(const float *cl, const float *m, const float *o, int C, int64_t N, int lerp,
                 float *y) {
    const int64_t n = (int64_t) C * N;
    if (lerp)
        run_flat(n, [&] { clsp_kernel<true>(cl, m, o, y, n, C, N); });
    else
        run_flat(n, [&] { clsp_kernel<false>(cl, m, nullptr, y, n, C, N); });
}

void ref_cu_flow_grid(const float *fl, const float *xs, int64_t N, float *y) {
    run_flat(3 * N, [&] { flow_grid_kernel(fl, xs, y, N); });
}

}  // extern "C"
