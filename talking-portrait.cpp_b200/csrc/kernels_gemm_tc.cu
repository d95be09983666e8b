// The library's plain GEMM on the tcgen05 tensor cores, for the sampler's
// linears (src/fmt.cpp:64-211) and the audio encoder's convolutions, linears
// and attention products (src/audio_enc.cpp:55-236):
//
//   Y[m][n] = epi( sum_k X[m][k] * W[n][k] ),  epi(v) = act((v + bias[n]) * scale) (+ res[m][n])
//
// both operands K-major (rows of X and of W run along k), f32 accumulation
// in tensor memory. A CTA owns a 128 x BN output tile: the 128 rows of W
// are the MMA's M side, BN rows of X its N side, so the accumulator lane is
// the output column n.
//
// Two arithmetic kinds:
//  * f16: f16 operands (kind::f16), as the reference's f16 mode runs its
//    linears (f16 weights and inputs, f32 accumulation);
//  * f32: float32 operands by the three-pass TF32 split (kind::tf32): each
//    operand x = hi + lo with hi = x rounded to TF32's 10 mantissa bits and
//    lo = x - hi (exact in f32), and a.b ~ hi_a.hi_b + hi_a.lo_b + lo_a.hi_b
//    (the "3xTF32" decomposition of Ootomo and Yokota, "Recovering single
//    precision accuracy from Tensor Cores while surpassing the FP32
//    theoretical peak", 2022). The split happens in shared memory: TMA lands
//    the raw f32 tile, the eight epilogue warps (idle in the main loop)
//    overwrite it with hi and write lo beside it, and the MMA warp issues the
//    three products. Relative error per product is about 2^-20.
//
// Batches (grid z) address their operands by row and column offsets into
// one 2-D view of each buffer (attention heads are column blocks of the
// q/k/v rows, grouped-conv groups are row blocks). Eight epilogue warps
// (two per TMEM lane quarter, each half of the columns) apply the epilogue
// into a shared-memory tile that one TMA store writes out (clipped to M and
// N per batch by the tensor map); outputs whose strides TMA cannot address
// take plain stores. Split-K, for grids with fewer tiles than SMs: the
// S <= 8 CTAs of a tile's K splits form one thread-block cluster (grid y);
// each leaves its partial accumulator in its own shared memory, and after a
// cluster barrier each CTA reads its column slice from all S CTAs
// (distributed shared memory), adds the partials in split order and stores
// it, so results do not depend on scheduling. Every pipeline wait is
// bounded; an expired wait sets *err and the CTA skips the rest of its work
// (it still takes part in the cluster barriers).
#include "tc_ptx.cuh"
#include "tpmd_internal.h"
#include "../../include/tpmd.h"

#include <algorithm>
#include <cstring>
#include <mutex>

namespace tpmd {
namespace {

constexpr int GK_F16 = 0, GK_TF32X3 = 1;

__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    const uint32_t mask = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(mask));
}

__device__ __forceinline__ float gelu_erf_g(float v) { return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f)); }
__device__ __forceinline__ float gelu_tanh_g(float v) {
    const float c = 0.7978845608028654f;  // sqrt(2/pi)
    return 0.5f * v * (1.0f + tanhf(c * (v + 0.044715f * v * v * v)));
}

template <int KIND, int BN>
struct gemm_cfg {
    static constexpr bool X3 = KIND == GK_TF32X3;
    static constexpr int ES = X3 ? 4 : 2;     // element bytes
    static constexpr int KB = 128 / ES;       // k elements per block (one 128-byte swizzled row)
    static constexpr int KSTEP = 32 / ES;     // k elements per MMA (32 bytes)
    static constexpr int A_BYTES = 128 * 128;
    static constexpr int B_BYTES = BN * 128;
    // raw (then hi) A and B, and with the split their lo halves
    static constexpr int STAGE_BYTES = (A_BYTES + B_BYTES) * (X3 ? 2 : 1);
    static constexpr int STAGE_TX = A_BYTES + B_BYTES;
    // f16: stages within ~100 KB so two CTAs share an SM; the split needs two
    static constexpr int STAGES_F16 = (102400 / STAGE_BYTES) > 6 ? 6 : (102400 / STAGE_BYTES);
    static constexpr int STAGES = X3 ? 2 : (STAGES_F16 < 2 ? 2 : STAGES_F16);
    static constexpr uint32_t TMEM_COLS = BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
    // D f32 (bit 4); A/B type f16 (0) or tf32 (2) at bits 7 and 10; K-major
    // both; N >> 3 at bit 17; M >> 4 at bit 24
    static constexpr uint32_t IDESC = (1u << 4) | ((X3 ? 2u : 0u) << 7) | ((X3 ? 2u : 0u) << 10) |
                                      ((uint32_t) (BN >> 3) << 17) | ((uint32_t) (128 >> 4) << 24);
    // the output tile [BN][128] (f32 at most) staged for the TMA store, or
    // the split-K partial, in the stage buffers once the main loop is done
    static constexpr int MAX_SPLITS = 8;
    static constexpr int OUT_BYTES = BN * 128 * 4;
    static constexpr int DATA_BYTES = STAGES * STAGE_BYTES > OUT_BYTES ? STAGES * STAGE_BYTES : OUT_BYTES;
    static constexpr int NEPI = 8;  // epilogue (and TF32 split) warps: 256 threads (named barrier 1)
    static constexpr int THREADS = 64 + 32 * NEPI;
    static constexpr int NBARS = 3 * STAGES + 1;
    static constexpr int SMEM = 1024 + DATA_BYTES + NBARS * 8 + 16;
    static_assert(BN % 16 == 0 && BN >= 64 && BN <= 256, "N tile");
    static_assert(SMEM <= 232448, "shared memory");
};

struct gemm_kparams {
    int M, N, K;
    int kblocks, kb_per_split, splits, tiles_n;
    int x_row_b, x_col_b, w_row_b, w_col_b;
    float *Y;
    __half *Yh;
    int64_t ldy, y_batch;
    const float *bias;
    float scale;
    int act;  // 0 none, 1 GELU (erf), 2 GELU (tanh), 3 leaky ReLU (0.2)
    const float *res;  // added after act, laid out as Y (may be Y itself)
    int y_tma;  // 0: plain stores; 2 / 3: the output tensor map's rank
    int y_vec;  // the output takes 4-element vector stores (aligned base and strides)
    int w_pre;  // W tiles loaded before the programmatic-dependence wait
    int *err;
};

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
__device__ __forceinline__ float4 ld_cluster_f32x4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *tm, uint32_t src, int c0, int c1) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     (uint64_t) tm),
                 "r"(src), "r"(c0), "r"(c1)
                 : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *tm, uint32_t src, int c0, int c1, int c2) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                     (uint64_t) tm),
                 "r"(src), "r"(c0), "r"(c1), "r"(c2)
                 : "memory");
}

// AND of v over the 256 epilogue threads (named barrier 1)
__device__ __forceinline__ bool epi_all(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, 1, 256, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t) v)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ float epi(float v, float bn, float scale, int act) {
    v = (v + bn) * scale;
    if (act == 1) v = gelu_erf_g(v);
    else if (act == 2) v = gelu_tanh_g(v);
    else if (act == 3) v = fmaxf(v, 0.2f * v);
    return v;
}

// x = hi + lo in place: hi (TF32-representable, round half away from zero
// at mantissa bit 13) overwrites x, lo = x - hi goes to `lo`
__device__ __forceinline__ void split_tf32(float4 *x, float4 *lo, int n4, int t, int nt) {
    for (int i = t; i < n4; i += nt) {
        float4 v = x[i], h, l;
        h.x = __uint_as_float((__float_as_uint(v.x) + 0x1000u) & 0xFFFFE000u);
        h.y = __uint_as_float((__float_as_uint(v.y) + 0x1000u) & 0xFFFFE000u);
        h.z = __uint_as_float((__float_as_uint(v.z) + 0x1000u) & 0xFFFFE000u);
        h.w = __uint_as_float((__float_as_uint(v.w) + 0x1000u) & 0xFFFFE000u);
        l.x = __fsub_rn(v.x, h.x);
        l.y = __fsub_rn(v.y, h.y);
        l.z = __fsub_rn(v.z, h.z);
        l.w = __fsub_rn(v.w, h.w);
        x[i] = h;
        lo[i] = l;
    }
}

template <int KIND, int BN>
__global__ void __launch_bounds__(gemm_cfg<KIND, BN>::THREADS, 2) gemm_tc_kernel(const __grid_constant__ CUtensorMap tmW,
                                                                             const __grid_constant__ CUtensorMap tmX,
                                                                             const __grid_constant__ CUtensorMap tmY,
                                                                             const gemm_kparams p) {
    using cfg = gemm_cfg<KIND, BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *) (((uintptr_t) smem_raw + 1023) & ~(uintptr_t) 1023);
    uint64_t *bars = (uint64_t *) (smem + cfg::DATA_BYTES);
    uint32_t *tmem_slot = (uint32_t *) (bars + cfg::NBARS);
    auto A = [&](int s) { return smem + s * cfg::STAGE_BYTES; };
    auto B = [&](int s) { return A(s) + cfg::A_BYTES; };
    auto Alo = [&](int s) { return A(s) + cfg::A_BYTES + cfg::B_BYTES; };
    auto Blo = [&](int s) { return Alo(s) + cfg::A_BYTES; };
    auto full = [&](int s) { return smem_u32(&bars[s]); };
    auto empty = [&](int s) { return smem_u32(&bars[cfg::STAGES + s]); };
    auto split_done = [&](int s) { return smem_u32(&bars[2 * cfg::STAGES + s]); };
    const uint32_t tfull = smem_u32(&bars[3 * cfg::STAGES]);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile = blockIdx.x, split = blockIdx.y, b = blockIdx.z;
    const int n0 = (tile % p.tiles_n) * 128, m0 = (tile / p.tiles_n) * BN;
    const int kb0 = split * p.kb_per_split;
    const int nk = min(p.kblocks - kb0, p.kb_per_split);  // >= 1 (host)

    if (threadIdx.x == 0) {
        for (int s = 0; s < cfg::STAGES; s++) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
            mbar_init(split_done(s), cfg::NEPI);
        }
        mbar_init(tfull, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(cfg::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;

    if (warp == 0) {
        if (lane == 0) {  // TMA producer
            // constant W: the first stages' W tiles before the wait on the
            // kernel before this one (which may still be running)
            const int pre = p.w_pre ? min(nk, cfg::STAGES) : 0;
            for (int i = 0; i < pre; i++) {
                mbar_expect_tx(full(i), cfg::STAGE_TX);
                tma_load_2d(smem_u32(A(i)), &tmW, full(i), (kb0 + i) * cfg::KB + b * p.w_col_b, n0 + b * p.w_row_b);
            }
            pdl_wait();
            pdl_trigger();
            int issued = 0;
            for (int i = 0; i < nk; i++) {
                const int s = i % cfg::STAGES;
                if (i >= cfg::STAGES && !mbar_wait(empty(s), ((i / cfg::STAGES) - 1) & 1)) {
                    ok = false;
                    break;
                }
                const int kc = (kb0 + i) * cfg::KB;
                if (i >= pre) {
                    mbar_expect_tx(full(s), cfg::STAGE_TX);
                    tma_load_2d(smem_u32(A(s)), &tmW, full(s), kc + b * p.w_col_b, n0 + b * p.w_row_b);
                }
                tma_load_2d(smem_u32(B(s)), &tmX, full(s), kc + b * p.x_col_b, m0 + b * p.x_row_b);
                issued++;
            }
            // W tiles issued before an early exit still land
            if (issued < pre) issued = pre;
            // the copies in flight land before the CTA goes on
            for (int j = issued > cfg::STAGES ? issued - cfg::STAGES : 0; j < issued; j++)
                if (!mbar_wait(full(j % cfg::STAGES), (j / cfg::STAGES) & 1)) ok = false;
            if (!ok) atomicExch(p.err, 1);
        }
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer
            for (int i = 0; i < nk; i++) {
                const int s = i % cfg::STAGES;
                if (!mbar_wait(cfg::X3 ? split_done(s) : full(s), (i / cfg::STAGES) & 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a = smem_u32(A(s)), bb = smem_u32(B(s));
#pragma unroll
                for (int kk = 0; kk < cfg::KB / cfg::KSTEP; kk++) {
                    const uint64_t ad = smem_desc(a + kk * 32, 1024, 2), bd = smem_desc(bb + kk * 32, 1024, 2);
                    const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
                    if constexpr (cfg::X3) {
                        const uint64_t adl = smem_desc(smem_u32(Alo(s)) + kk * 32, 1024, 2);
                        const uint64_t bdl = smem_desc(smem_u32(Blo(s)) + kk * 32, 1024, 2);
                        umma_tf32(tmem, ad, bd, cfg::IDESC, acc);
                        umma_tf32(tmem, ad, bdl, cfg::IDESC, 1u);
                        umma_tf32(tmem, adl, bd, cfg::IDESC, 1u);
                    } else {
                        umma_f16(tmem, ad, bd, cfg::IDESC, acc);
                    }
                }
                umma_commit(empty(s));
            }
            if (ok) umma_commit(tfull);
            else atomicExch(p.err, 1);
        }
    } else {
        // warps 2..9: the TF32 split of each stage, then the epilogue
        const int et = threadIdx.x - 64;
        if constexpr (cfg::X3) {
            for (int i = 0; i < nk; i++) {
                const int s = i % cfg::STAGES;
                if (!mbar_wait(full(s), (i / cfg::STAGES) & 1)) {
                    ok = false;
                    break;
                }
                split_tf32((float4 *) A(s), (float4 *) Alo(s), cfg::A_BYTES / 16, et, 32 * cfg::NEPI);
                split_tf32((float4 *) B(s), (float4 *) Blo(s), cfg::B_BYTES / 16, et, 32 * cfg::NEPI);
                // generic-proxy writes before the tensor core's async-proxy reads
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(split_done(s));
            }
        }
        if (ok && !mbar_wait(tfull, 0)) ok = false;
        // uniform over the epilogue warps: tcgen05.ld is warp-collective and
        // the TMA store waits on the epilogue's named barrier
        ok = epi_all(ok);
        pdl_wait();  // (returned long ago in the producer) before any global write
        if (!ok) {
            if (et == 0) atomicExch(p.err, 1);
        } else {
            tc_fence_after();
            // lane quarter q of TMEM (row n0 + row), columns [c_lo, c_lo + BN/2)
            const int q = warp & 3, row = q * 32 + lane, n = n0 + row;
            const int c_lo = ((warp - 2) >> 2) * (BN / 2);
            const uint32_t taddr = tmem + ((uint32_t) (q * 32) << 16);
            float *sf = (float *) smem;  // [BN][128]: the output tile for the TMA store
            __half *sh = (__half *) smem;
            const float bn = (p.splits == 1 && p.bias && n < p.N) ? __ldg(p.bias + n) : 0.0f;
            const bool plain = p.splits == 1 && !p.y_tma;
            float *yp = nullptr;
            __half *yhp = nullptr;
            if (plain) {
                const int64_t o = (int64_t) b * p.y_batch + (int64_t) (m0 + c_lo) * p.ldy + n;
                if (p.Yh) yhp = p.Yh + o;
                else yp = p.Y + o;
            }
            const int mlim = p.M - m0;
#pragma unroll 1
            for (int c = c_lo; p.splits == 1 && c < c_lo + BN / 2 && c < mlim; c += 16) {
                uint32_t r[16];
                tmem_ld16(taddr + c, r);
                if (!plain) {
                    if (p.Yh) {
#pragma unroll
                        for (int j = 0; j < 16; j++)
                            sh[(c + j) * 128 + row] = __float2half_rn(epi(__uint_as_float(r[j]), bn, p.scale, p.act));
                    } else if (p.res) {
                        // the residual of rows inside the output only (the rest is clipped)
                        const float *rp = p.res + (int64_t) b * p.y_batch + (int64_t) (m0 + c) * p.ldy + n;
#pragma unroll
                        for (int j = 0; j < 16; j++)
                            sf[(c + j) * 128 + row] = epi(__uint_as_float(r[j]), bn, p.scale, p.act) +
                                                      ((n < p.N && c + j < mlim) ? rp[(int64_t) j * p.ldy] : 0.0f);
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; j++)
                            sf[(c + j) * 128 + row] = epi(__uint_as_float(r[j]), bn, p.scale, p.act);
                    }
                } else if (n < p.N) {
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        if (c + j < mlim) {
                            const int64_t o = (int64_t) (c - c_lo + j) * p.ldy;
                            float v = epi(__uint_as_float(r[j]), bn, p.scale, p.act);
                            if (yhp) {
                                yhp[o] = __float2half_rn(v);
                            } else {
                                if (p.res) v += p.res[(yp - p.Y) + o];
                                yp[o] = v;
                            }
                        }
                    }
                }
            }
            if (p.splits == 1 && p.y_tma) {
                // the tile to global memory by one TMA store (clipped to M, N)
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                asm volatile("bar.sync 1, 256;" ::: "memory");
                if (et == 0) {
                    if (p.y_tma == 3) tma_store_3d(&tmY, smem_u32(smem), n0, m0, b);
                    else tma_store_2d(&tmY, smem_u32(smem), n0, m0);
                    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
                }
            }
        }
    }
    if (p.splits > 1) {
        // split-K over the cluster: every CTA leaves its partial [BN][128]
        // in its own shared memory; after a cluster barrier CTA `split` adds
        // columns [c0, c1) of all S partials in split order (distributed
        // shared memory reads, four rows per 16-byte load; thread: rows
        // 4 rq .. 4 rq + 3, columns c0 + cl + 8 i, two columns per round)
        const int S = p.splits, W = (BN + S - 1) / S;
        if (warp >= 2 && ok) {
            const int q = warp & 3, row = q * 32 + lane;
            const int c_lo = ((warp - 2) >> 2) * (BN / 2);
            const uint32_t taddr = tmem + ((uint32_t) (q * 32) << 16);
            float *part = (float *) smem;
#pragma unroll 1
            for (int c = c_lo; c < c_lo + BN / 2; c += 16) {
                uint32_t r[16];
                tmem_ld16(taddr + c, r);
#pragma unroll
                for (int j = 0; j < 16; j++) part[(c + j) * 128 + row] = __uint_as_float(r[j]);
            }
        }
        __syncwarp();
        cluster_sync_all();
        if (warp >= 2 && ok) {
            const int et = threadIdx.x - 64;
            const int rq = et & 31, cl = et >> 5;
            const int nq = n0 + 4 * rq;
            const int c0 = split * W, c1 = min(min(BN, c0 + W), p.M - m0);
            uint32_t src[cfg::MAX_SPLITS];
            const uint32_t mine = smem_u32(smem) + (uint32_t) rq * 16u;
#pragma unroll
            for (int s2 = 0; s2 < cfg::MAX_SPLITS; s2++) src[s2] = s2 < S ? map_to_rank(mine, (uint32_t) s2) : 0u;
            float bq[4];
#pragma unroll
            for (int e = 0; e < 4; e++) bq[e] = (p.bias && nq + e < p.N) ? __ldg(p.bias + nq + e) : 0.0f;
            const int64_t ybase = (int64_t) b * p.y_batch;
            const bool full4 = nq + 3 < p.N;
            for (int cb = c0 + cl; cb < c1; cb += 16) {
                // columns cb and cb + 8: all their loads in flight together
                float4 pv[2][cfg::MAX_SPLITS];
#pragma unroll
                for (int u = 0; u < 2; u++)
#pragma unroll
                    for (int s2 = 0; s2 < cfg::MAX_SPLITS; s2++)
                        if (s2 < S && cb + 8 * u < c1) pv[u][s2] = ld_cluster_f32x4(src[s2] + (uint32_t) (cb + 8 * u) * 512u);
#pragma unroll
                for (int u = 0; u < 2; u++) {
                    const int c = cb + 8 * u;
                    if (c >= c1) break;
                    float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                    for (int s2 = 0; s2 < cfg::MAX_SPLITS; s2++)
                        if (s2 < S) {
                            v[0] += pv[u][s2].x;
                            v[1] += pv[u][s2].y;
                            v[2] += pv[u][s2].z;
                            v[3] += pv[u][s2].w;
                        }
#pragma unroll
                    for (int e = 0; e < 4; e++) v[e] = epi(v[e], bq[e], p.scale, p.act);
                    const int64_t o = ybase + (int64_t) (m0 + c) * p.ldy + nq;
                    if (p.res && !p.Yh) {
#pragma unroll
                        for (int e = 0; e < 4; e++)
                            if (nq + e < p.N) v[e] += p.res[o + e];
                    }
                    if (p.y_vec && full4) {
                        if (p.Yh) {
                            __half2 h01 = __floats2half2_rn(v[0], v[1]), h23 = __floats2half2_rn(v[2], v[3]);
                            uint2 w2;
                            w2.x = *(uint32_t *) &h01;
                            w2.y = *(uint32_t *) &h23;
                            *(uint2 *) (p.Yh + o) = w2;
                        } else {
                            *(float4 *) (p.Y + o) = make_float4(v[0], v[1], v[2], v[3]);
                        }
                    } else {
#pragma unroll
                        for (int e = 0; e < 4; e++)
                            if (nq + e < p.N) {
                                if (p.Yh) p.Yh[o + e] = __float2half_rn(v[e]);
                                else p.Y[o + e] = v[e];
                            }
                    }
                }
            }
        }
        __syncwarp();
        cluster_sync_all();  // no CTA leaves while others read its partial
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(cfg::TMEM_COLS)
                     : "memory");
}

bool encode_2d(CUtensorMap *tm, bool f32, const void *base, int64_t cols, int64_t rows, int64_t ld, int box_cols,
               int box_rows) {
    auto enc = encode_fn();
    if (!enc) return false;
    const int es = f32 ? 4 : 2;
    const cuuint64_t dims[2] = {(cuuint64_t) cols, (cuuint64_t) rows};
    const cuuint64_t strides[1] = {(cuuint64_t) (ld * es)};
    const cuuint32_t box[2] = {(cuuint32_t) box_cols, (cuuint32_t) box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(tm, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void *) base, dims,
               strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int KIND, int BN>
cudaError_t set_smem_attr() {
    static uint64_t attr_set = 0;  // one bit per device
    static std::mutex mu;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> g(mu);
    if (attr_set >> (dev & 63) & 1) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<KIND, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               gemm_cfg<KIND, BN>::SMEM);
    if (e == cudaSuccess) attr_set |= 1ull << (dev & 63);
    return e;
}

template <int KIND, int BN>
cudaError_t run_gemm(const gemm_desc &d, cudaStream_t st) {
    using cfg = gemm_cfg<KIND, BN>;
    gemm_kparams p{};
    p.M = d.M;
    p.N = d.N;
    p.K = d.K;
    p.kblocks = (d.K + cfg::KB - 1) / cfg::KB;
    p.tiles_n = (d.N + 127) / 128;
    const int tiles_m = (d.M + BN - 1) / BN;
    const int64_t tiles = (int64_t) p.tiles_n * tiles_m;
    if (tiles >= (1 << 30) || d.batch > 65535) return cudaErrorInvalidValue;
    // column-offset batches read whole k-blocks inside their own columns
    if ((d.x_col_b || d.w_col_b) && d.K % cfg::KB) return cudaErrorInvalidValue;
    // split K until the grid covers the SMs (a cluster of at most 8 CTAs per
    // tile), keeping >= 2 k-blocks per split
    int splits = 1;
    const int64_t ctas = tiles * d.batch;
    if (ctas < sm_count()) {
        splits = (int) ((sm_count() + ctas - 1) / ctas);
        splits = std::min(splits, std::max(1, p.kblocks / 2));
        splits = std::min(splits, cfg::MAX_SPLITS);
    }
    p.kb_per_split = (p.kblocks + splits - 1) / splits;
    p.splits = (p.kblocks + p.kb_per_split - 1) / p.kb_per_split;  // no empty split
    p.x_row_b = d.x_row_b;
    p.x_col_b = d.x_col_b;
    p.w_row_b = d.w_row_b;
    p.w_col_b = d.w_col_b;
    p.Y = d.Y;
    p.Yh = d.Yh;
    p.ldy = d.ldy;
    p.y_batch = d.y_batch;
    p.bias = d.bias;
    p.scale = d.scale;
    p.act = d.act;
    p.res = d.res;
    p.err = d.err;
    p.w_pre = d.pdl && d.w_const;
    CUtensorMap tmW, tmX, tmY;
    memset(&tmY, 0, sizeof tmY);
    {
        const int eo = d.Yh ? 2 : 4;
        const uintptr_t yb = d.Yh ? (uintptr_t) d.Yh : (uintptr_t) d.Y;
        p.y_vec = !(yb & (uintptr_t) (4 * eo - 1)) && d.ldy % 4 == 0 && (d.batch == 1 || d.y_batch % 4 == 0);
    }
    p.y_tma = 0;
    if (splits == 1) {
        // the output by TMA where its strides allow: [batch][M][N], clipped
        const int eo = d.Yh ? 2 : 4;
        const void *yb = d.Yh ? (const void *) d.Yh : (const void *) d.Y;
        auto enc = encode_fn();
        if (enc && !((uintptr_t) yb & 15) && (d.ldy * eo) % 16 == 0 && (d.batch == 1 || (d.y_batch * eo) % 16 == 0)) {
            const CUtensorMapDataType ty = d.Yh ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
            const cuuint64_t dims[3] = {(cuuint64_t) d.N, (cuuint64_t) d.M, (cuuint64_t) d.batch};
            const cuuint64_t strides[2] = {(cuuint64_t) (d.ldy * eo), (cuuint64_t) (d.y_batch * eo)};
            const cuuint32_t box[3] = {128, (cuuint32_t) BN, 1};
            const cuuint32_t estr[3] = {1, 1, 1};
            const int rank = d.batch == 1 ? 2 : 3;
            if (enc(&tmY, ty, rank, (void *) yb, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS)
                p.y_tma = rank;
        }
    }
    const bool f32 = cfg::X3;
    const int64_t xrows = (int64_t) (d.batch - 1) * d.x_row_b + d.M, xcols = (int64_t) (d.batch - 1) * d.x_col_b + d.K;
    const int64_t wrows = (int64_t) (d.batch - 1) * d.w_row_b + d.N, wcols = (int64_t) (d.batch - 1) * d.w_col_b + d.K;
    if (!encode_2d(&tmW, f32, d.W, wcols, wrows, d.ldw, cfg::KB, 128) ||
        !encode_2d(&tmX, f32, d.X, xcols, xrows, d.ldx, cfg::KB, BN))
        return cudaErrorInvalidValue;
    const cudaError_t ae = set_smem_attr<KIND, BN>();
    if (ae != cudaSuccess) return ae;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((unsigned) tiles, (unsigned) p.splits, (unsigned) d.batch);
    lc.blockDim = dim3(cfg::THREADS, 1, 1);
    lc.dynamicSmemBytes = cfg::SMEM;
    lc.stream = st;
    cudaLaunchAttribute at[2];
    int na = 0;
    if (p.splits > 1) {
        at[na].id = cudaLaunchAttributeClusterDimension;
        at[na].val.clusterDim.x = 1;
        at[na].val.clusterDim.y = (unsigned) p.splits;
        at[na].val.clusterDim.z = 1;
        na++;
    }
    if (d.pdl) {
        at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[na].val.programmaticStreamSerializationAllowed = 1;
        na++;
    }
    lc.attrs = at;
    lc.numAttrs = na;
    const cudaError_t le = cudaLaunchKernelEx(&lc, gemm_tc_kernel<KIND, BN>, tmW, tmX, tmY, p);
    return le != cudaSuccess ? le : cudaGetLastError();
}

template <int KIND>
cudaError_t run_kind(const gemm_desc &d, cudaStream_t st) {
    // the narrowest N tile that holds M; past 256 the one wasting fewer rows
    int bn;
    if (d.M <= 64) bn = 64;
    else if (d.M <= 128) bn = 128;
    else if (d.M <= 192) bn = 192;
    else if (d.M <= 256) bn = 256;
    else bn = ((d.M + 255) / 256) * 256 - d.M <= ((d.M + 191) / 192) * 192 - d.M ? 256 : 192;
    // grids too small for the SMs split K over a cluster; 64-wide N tiles
    // there give more CTAs, fewer splits and smaller partials to add
    const int64_t tiles = (int64_t) ((d.N + 127) / 128) * ((d.M + bn - 1) / bn) * d.batch;
    if (bn > 64 && tiles < sm_count()) bn = 64;
    switch (bn) {
        case 64: return run_gemm<KIND, 64>(d, st);
        case 128: return run_gemm<KIND, 128>(d, st);
        case 192: return run_gemm<KIND, 192>(d, st);
        default: return run_gemm<KIND, 256>(d, st);
    }
}

}  // namespace

cudaError_t gemm_tc_prepare() {
    cudaError_t e = cudaSuccess;
    for (cudaError_t r : {set_smem_attr<GK_F16, 64>(), set_smem_attr<GK_F16, 128>(), set_smem_attr<GK_F16, 192>(),
                          set_smem_attr<GK_F16, 256>(), set_smem_attr<GK_TF32X3, 64>(),
                          set_smem_attr<GK_TF32X3, 128>(), set_smem_attr<GK_TF32X3, 192>(),
                          set_smem_attr<GK_TF32X3, 256>()})
        if (r != cudaSuccess) e = r;
    return e;
}

cudaError_t gemm_tc(const gemm_desc &d, cudaStream_t st) {
    const int es = d.f32 ? 4 : 2;
    if (d.M <= 0 || d.N <= 0 || d.K <= 0 || d.batch <= 0 || !d.X || !d.W || (!d.Y == !d.Yh) || !d.err)
        return cudaErrorInvalidValue;
    // TMA: 16-byte aligned bases and row strides
    if (((uintptr_t) d.X | (uintptr_t) d.W) & 15 || (d.ldx * es) % 16 || (d.ldw * es) % 16 || d.ldx < d.K ||
        d.ldw < d.K || d.ldy < d.N || d.act < 0 || d.act > 3 || (d.res && d.Yh))
        return cudaErrorInvalidValue;
    if (d.batch > 1 && (d.x_row_b < 0 || d.x_col_b < 0 || d.w_row_b < 0 || d.w_col_b < 0 || d.y_batch < 0))
        return cudaErrorInvalidValue;
    return d.f32 ? run_kind<GK_TF32X3>(d, st) : run_kind<GK_F16>(d, st);
}

}  // namespace tpmd

namespace {
// tpk_gemm's error flag, one per device
std::mutex g_flag_mu;
int *g_flag[64];
}  // namespace

extern "C" int tpk_gemm(const void *X, int64_t ldx, const void *W, int64_t ldw, float *Y, int64_t ldy, int M, int N,
                        int K, int batch, int x_row_b, int x_col_b, int w_row_b, int w_col_b, int64_t y_batch,
                        int dtype, const float *bias, float scale, int act, void *stream) {
    using namespace tpmd;
    if (dtype != TPMD_DTYPE_F32 && dtype != TPMD_DTYPE_F16) return tpk_fail("tpk_gemm: dtype");
    if (act < 0 || act > 3) return tpk_fail("tpk_gemm: act");
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return tpk_fail("tpk_gemm: no device");
    int *flag_d = nullptr;
    {
        std::lock_guard<std::mutex> g(g_flag_mu);
        if (!g_flag[dev]) {
            if (cudaMalloc(&g_flag[dev], sizeof(int)) != cudaSuccess ||
                cudaMemset(g_flag[dev], 0, sizeof(int)) != cudaSuccess) {
                cudaGetLastError();
                if (g_flag[dev]) cudaFree(g_flag[dev]);
                g_flag[dev] = nullptr;
                return tpk_fail("tpk_gemm: allocation failed");
            }
        }
        flag_d = g_flag[dev];
    }
    cudaStream_t st = (cudaStream_t) stream;
    gemm_desc d;
    d.f32 = dtype == TPMD_DTYPE_F32;
    d.X = X;
    d.ldx = ldx;
    d.W = W;
    d.ldw = ldw;
    d.Y = Y;
    d.ldy = ldy;
    d.y_batch = y_batch;
    d.M = M;
    d.N = N;
    d.K = K;
    d.batch = batch;
    d.x_row_b = x_row_b;
    d.x_col_b = x_col_b;
    d.w_row_b = w_row_b;
    d.w_col_b = w_col_b;
    d.bias = bias;
    d.scale = scale;
    d.act = act;
    d.err = flag_d;
    cudaError_t e = gemm_tc(d, st);
    if (e == cudaErrorInvalidValue) return tpk_fail("tpk_gemm: bad shape, stride or alignment");
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return tpk_fail(std::string("tpk_gemm: ") + cudaGetErrorString(e));
    }
    int flag = 0;
    if (cudaMemcpy(&flag, d.err, sizeof flag, cudaMemcpyDeviceToHost) != cudaSuccess)
        return tpk_fail("tpk_gemm: status read failed");
    if (flag) {
        cudaMemset(d.err, 0, sizeof(int));
        return tpk_fail("tpk_gemm: a pipeline wait timed out");
    }
    return 0;
}
