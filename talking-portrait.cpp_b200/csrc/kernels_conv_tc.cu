// Modulated 3x3 conv as a tcgen05 implicit GEMM (f16 in, f32 accumulate in
// TMEM, f16 out) for sm_100a.
//
// GEMM view (as the SIMT kernel): M = input-grid pixels of the batch, N = OC
// (dense) or 4*OC (sub-pixel up-conv: the conv_transpose+blur composition of
// src/motion_dec.cpp:144-191 as four parity classes), K = 9*IC in the order
// k = tap*IC + ic.
//
// Structure (one CTA per SM, persistent over tiles of 128 pixels x BN columns):
//  * warp 0, one lane: TMA producer. Per k-step it loads the A tile as ONE
//    4-D box {KC channels, bw, bh, bb} of the channel-last activation at the
//    tap's shifted coordinates (x-1..x+1, y-1..y+1); TMA's zero fill of the
//    out-of-range part IS the conv's padding, so no im2col buffer exists. The
//    B tile is a 2-D box {KC, BN} of the [N][K] weight matrix. Both land in
//    shared memory in the 128-byte (KC = 64) or 64-byte (KC = 32) swizzled
//    K-major layout that tcgen05 descriptors address directly.
//  * warp 1, one lane: issues tcgen05.mma (M=128, N=BN, K=16) into a TMEM
//    accumulator, commits each stage back to the producer and each finished
//    tile to the epilogue. Two accumulators (2*BN TMEM columns) let the
//    epilogue of tile t overlap the MMAs of tile t+1.
//  * warps 2-5: epilogue. Each warp reads its 32-lane quarter of TMEM
//    (tcgen05.ld 32x32b), applies x inv_den[b][o] (demodulation with the
//    FusedLeakyReLU gain folded), + bias, leaky ReLU 0.2, x the next conv's
//    style, and stores f16 channel-last rows (sub-pixel scatter for the up-conv).
// Every mbarrier wait is bounded (~2 s of %globaltimer); on expiry the kernel
// sets *err, stops issuing work, waits (bounded) for its own copies and MMAs
// in flight, frees its TMEM and returns.
#include "tc_ptx.cuh"
#include "tpmd_internal.h"

namespace tpmd {
namespace {

constexpr int BM = 128;

struct tc_params {
    int B, H, W, IC, OC, N;
    int kiters, cpt;           // k-steps per tile, channel chunks per tap
    int bw, bh, bb;            // pixel box of one M tile
    int tiles_x, tiles_y, tiles_n;
    int lg_x, lg_y, lg_n;      // their log2
    int lg_oc;                 // log2 of OC (sub-pixel class of column n = n >> lg_oc)
    int num_tiles;
    int yb, strips;            // KHS: output rows per work unit, units per column of the map
    __half *y;
    const float *inv_den;
    int den_stride;
    const float *bias;
    const float *snext;
    int snext_stride;
    int *err;
    long long stall_ns;  // test hook: wait this long on a barrier nothing completes, then abort
    // fused level tail (conv2 kernels of the levels with OC <= 256)
    const __half *feat;
    const float *fW, *fs;
    int s_stride;
    const float *fb, *fup, *skipf_prev;
    float *skipf_out;
    const float *rW, *rlb, *rb, *rup, *skip_prev;
    float *skip_out;
    const float *lin;
    __half *trunk;
    const float *tsn;  // next up-conv style, multiplied into the trunk
    const float4 *proj;  // last level: ToRGB conv.0 applied to the feats per pixel
};

template <int BN, int KC, int NACC, bool TAIL, bool BRES, bool HALO = false, int RPS = 1, bool KHS = false,
          bool DEEP = false>
struct tc_cfg {
    static constexpr int A_TAP = BM * KC * 2;   // one tap's A tile
    static constexpr int B_TAP = BN * KC * 2;   // one tap's B tile
    // HALO: a tile is one 128-pixel row; per kernel row one TMA box of the
    // 130 pixels x-1..x+128 serves all three horizontal taps, each tap's A
    // operand being the same box started 0, 1 or 2 rows later (a descriptor
    // offset; swizzling follows absolute shared addresses). 136 rows are
    // reserved per box to keep the next box 1024-byte aligned.
    static constexpr int HALO_ROWS = BM + 2;
    static constexpr int A_HALO = 136 * KC * 2;
    // fused tail: the ToFlow weights [3][BN] and the two up-sampling kernels,
    // shared by all epilogue groups, then per epilogue group two buffers
    // (alternating by tile) of the tile's per-frame channel constants:
    // inv_den, bias, the three ToFlow weights times the ToFlow style, and
    // the next up-conv's style (CW floats)
    // Staged only for tiles of at most 128 channels (r128, r256, r512): at
    // BN = 256 (r64) the per-pixel loads of the old form measured faster
    static constexpr bool STG = TAIL && BN <= 128;
    static constexpr int CW = 6 * BN;
    // XCH (levels with a trunk, BN >= 64): the trunk pass gathers the feats
    // cooperatively, four lanes per 32-channel slice of a pixel's tap row,
    // through a per-warp exchange area of eight pixels' activations (8 rows
    // of 36 floats, padded against bank conflicts) and tap geometry (8 rows
    // of 12 words). Used at 64 and 128 channels (r256, r128), where it
    // measured faster; the 256-channel r64 tile keeps the per-pixel pass
    static constexpr bool XCH = TAIL && (BN == 64 || BN == 128);
    static constexpr int XW = 8 * 36 + 8 * 12;  // floats per epilogue warp
    static constexpr int EXTRA =
        TAIL ? (3 * BN + 32 + (STG ? NACC * 2 * CW : 0) + (XCH ? 4 * NACC * XW : 0)) * 4 : 0;
    // BRES: the whole weight matrix (9 taps x one KC chunk) stays resident in
    // shared memory for the kernel's lifetime instead of being re-loaded for
    // every pixel tile; stages then carry only A
    static constexpr int B_RES = BRES ? 9 * B_TAP : 0;
    // XCH configurations count the dynamic shared memory exactly (less the
    // alignment pad and a bound on the barriers); the others keep the
    // earlier cap
    static constexpr int BUDGET = XCH ? 232448 - 1024 - 640 - EXTRA - B_RES : 212992 - EXTRA - B_RES;
    // taps per pipeline stage: narrow layers put a whole kernel row (3 taps)
    // in one stage, so the per-stage barrier round trip is paid 3x less often
    // DEEP: one tap per stage regardless of width, for layers with fewer
    // tiles than SMs, whose CTAs each stream a long K (conv1, the r8 level):
    // six 32 KB stages in flight hide the load latency that two 96 KB stages
    // leave exposed
    static constexpr int TPS =
        HALO ? 3 : BRES ? (BUDGET / (3 * A_TAP) >= 3 ? 3 : 1) : (BN <= 128 && !DEEP ? 3 : 1);
    // RPS: kernel rows per stage (HALO with resident weights only); a stage
    // then holds RPS halo boxes and TAPS = 3 * RPS taps, fewer commits per tile
    static constexpr int TAPS = HALO ? 3 * RPS : TPS;
    static constexpr int A_BYTES = HALO ? RPS * A_HALO : TPS * A_TAP;     // per stage (space)
    static constexpr int A_TX = HALO ? RPS * HALO_ROWS * KC * 2 : A_BYTES;  // per stage (loaded)
    static constexpr int B_BYTES = BRES ? 0 : TAPS * B_TAP;  // per stage
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGE_TX = A_TX + B_BYTES;
    // as deep as shared memory allows (small stages hide more TMA latency)
    // an even count: stages are released to the producer in pairs (one
    // tcgen05.commit per two stages)
    static constexpr int STAGES = ((BUDGET / STAGE_BYTES) > 20 ? 20 : (BUDGET / STAGE_BYTES)) & ~1;
    static constexpr int B_REGION = BRES ? B_RES : STAGES * B_BYTES;
    // KHS (kernel rows stacked in N): a work unit is a strip of output rows of
    // one 128-pixel column segment; each input row is one halo box, multiplied
    // by the three kernel rows' weights side by side (N = 3 BN). Block j of
    // the product belongs to output row yi - 1 + j, so the accumulators of
    // consecutive output rows live in a ring of R = 512 / BN TMEM slots and
    // each output row is complete after the next input row. Slots are zeroed
    // by the epilogue after use, so every MMA accumulates.
    static constexpr int R = KHS ? 512 / BN : 0;
    static constexpr int NSLOT = KHS ? R : NACC;  // accumulators with their own full/empty barriers
    static constexpr uint32_t TMEM_COLS = KHS ? 512 : NACC * BN;  // one accumulator per epilogue group
    static constexpr int THREADS = 64 + 128 * NACC;
    static constexpr uint32_t LAYOUT = KC == 64 ? 2u : 4u;
    static constexpr uint32_t SBO = KC == 64 ? 1024u : 512u;
    // kind::f16 instruction descriptor: D f32, A/B f16, both K-major, N, M
    static constexpr uint32_t IDESC =
        (1u << 4) | ((uint32_t) (BN >> 3) << 17) | ((uint32_t) (BM >> 4) << 24);
    // the same with N = nb * BN (KHS: nb stacked kernel rows)
    static __device__ __forceinline__ uint32_t idesc_n(int nb) {
        return (1u << 4) | ((uint32_t) ((nb * BN) >> 3) << 17) | ((uint32_t) (BM >> 4) << 24);
    }
    // + per epilogue group one barrier for its staged constants (TAIL)
    static constexpr int NBARS = 2 * STAGES + 2 * NSLOT + 2 + NACC;
    static constexpr int SMEM = 1024 + STAGES * A_BYTES + B_REGION + EXTRA + NBARS * 8 + 16;
    static_assert((TMEM_COLS & (TMEM_COLS - 1)) == 0 && TMEM_COLS >= 32 && TMEM_COLS <= 512, "TMEM");
    static_assert(SMEM <= 232448, "shared memory");
    static_assert(STAGES >= 2, "pipeline depth");
    static_assert(RPS == 1 || (RPS == 3 && HALO && BRES), "rows per stage");
    static_assert(!KHS || (TAIL && HALO && BRES && RPS == 1 && (BN == 32 || BN == 64) && R % NACC == 0),
                  "stacked kernel rows");
};

struct tile_pos {
    int n0, b0, y0, x0;
};
// tile counts along n, x and y are powers of two (log2 in lg_*)
__device__ __forceinline__ tile_pos tile_of(const tc_params &p, int t, int BN) {
    tile_pos r;
    const int nt = t & (p.tiles_n - 1);
    const int m = t >> p.lg_n;
    const int xt = m & (p.tiles_x - 1);
    const int m2 = m >> p.lg_x;
    const int yt = m2 & (p.tiles_y - 1);
    const int bt = m2 >> p.lg_y;
    r.n0 = nt * BN;
    r.x0 = xt * p.bw;
    r.y0 = yt * p.bh;
    r.b0 = bt * p.bb;
    return r;
}

// 16 consecutive floats (64-byte aligned) through the read-only path
__device__ __forceinline__ void ld_f16x(const float *p, float *v) {
    const float4 *q = reinterpret_cast<const float4 *>(p);
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const float4 u = __ldg(q + j);
        v[4 * j] = u.x;
        v[4 * j + 1] = u.y;
        v[4 * j + 2] = u.z;
        v[4 * j + 3] = u.w;
    }
}

__device__ __forceinline__ void ld_half16(const __half *p, float *v) {
    const uint4 *q = reinterpret_cast<const uint4 *>(p);
#pragma unroll
    for (int j = 0; j < 2; j++) {
        const uint4 u = __ldg(q + j);
        const __half2 *h = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const float2 f = __half22float2(h[k]);
            v[8 * j + 2 * k] = f.x;
            v[8 * j + 2 * k + 1] = f.y;
        }
    }
}
__device__ __forceinline__ void st_half16(__half *p, const float *v) {
    uint4 pk[2];
    __half2 *h2 = reinterpret_cast<__half2 *>(pk);
#pragma unroll
    for (int i = 0; i < 8; i++) h2[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
    uint4 *q = reinterpret_cast<uint4 *>(p);
    q[0] = pk[0];
    q[1] = pk[1];
}

// 8 consecutive f16 values (16-byte aligned) as floats, and back
__device__ __forceinline__ void ld_half8(const __half *p, float *v) {
    const uint4 u = __ldg(reinterpret_cast<const uint4 *>(p));
    const __half2 *h = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const float2 f = __half22float2(h[k]);
        v[2 * k] = f.x;
        v[2 * k + 1] = f.y;
    }
}
__device__ __forceinline__ void st_half8(__half *p, const float *v) {
    uint4 q;
    __half2 *h2 = reinterpret_cast<__half2 *>(&q);
#pragma unroll
    for (int i = 0; i < 4; i++) h2[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4 *>(p) = q;
}

// KHS work unit t: (frame, strip of p.yb output rows, 128-pixel segment)
__device__ __forceinline__ void unit_of(const tc_params &p, int t, int &b, int &y0, int &x0) {
    const int xs = t % p.tiles_x, m = t / p.tiles_x;
    x0 = xs * BM;
    y0 = (m % p.strips) * p.yb;
    b = m / p.strips;
}

template <int BN, int KC, bool UP, int NACC, bool TAIL, bool BRES, bool HALO, int RPS, bool KHS, bool DEEP>
__global__ void __launch_bounds__(tc_cfg<BN, KC, NACC, TAIL, BRES, HALO, RPS, KHS, DEEP>::THREADS, 1)
conv_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const tc_params p) {
    using cfg = tc_cfg<BN, KC, NACC, TAIL, BRES, HALO, RPS, KHS, DEEP>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *) (((uintptr_t) smem_raw + 1023) & ~(uintptr_t) 1023);
    uint8_t *sA = smem;
    uint8_t *sB = smem + cfg::STAGES * cfg::A_BYTES;
    float *sx = (float *) (sB + cfg::B_REGION);  // TAIL constants
    uint64_t *bars = (uint64_t *) (sB + cfg::B_REGION + cfg::EXTRA);
    uint32_t *tmem_slot = (uint32_t *) (bars + cfg::NBARS);
    auto full = [&](int s) { return smem_u32(&bars[s]); };
    // per stage pair (KHS: per stage)
    auto empty = [&](int s) { return smem_u32(&bars[cfg::STAGES + (KHS ? s : (s >> 1))]); };
    auto tfull = [&](int a) { return smem_u32(&bars[2 * cfg::STAGES + a]); };
    auto tempty = [&](int a) { return smem_u32(&bars[2 * cfg::STAGES + cfg::NSLOT + a]); };
    const uint32_t drain = smem_u32(&bars[2 * cfg::STAGES + 2 * cfg::NSLOT]);
    const uint32_t bres_bar = smem_u32(&bars[2 * cfg::STAGES + 2 * cfg::NSLOT + 1]);
    auto cbar = [&](int g) { return smem_u32(&bars[2 * cfg::STAGES + 2 * cfg::NSLOT + 2 + g]); };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < cfg::STAGES; s++) {
            mbar_init(full(s), 1);
            if (KHS || !(s & 1)) mbar_init(empty(s), 1);
        }
        for (int a = 0; a < cfg::NSLOT; a++) {
            mbar_init(tfull(a), 1);
            mbar_init(tempty(a), 4);
        }
        mbar_init(drain, 1);
        mbar_init(bres_bar, 1);
        for (int g = 0; g < NACC; g++) mbar_init(cbar(g), 128);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (TAIL) {  // sx[0..3BN): ToFlow weights, then the flow and rgb up-sampling kernels
        for (int i = threadIdx.x; i < 3 * BN; i += blockDim.x) sx[i] = __ldg(p.fW + i);
        for (int i = threadIdx.x; i < 16; i += blockDim.x) {
            sx[3 * BN + i] = __ldg(p.fup + i);
            sx[3 * BN + 16 + i] = __ldg(p.rup + i);
        }
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(cfg::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    if constexpr (KHS) {
        // every ring slot starts at zero: the first epilogue group clears TMEM
        if (warp >= 2 && warp < 6) {
            const uint32_t lanes = (uint32_t) ((warp & 3) * 32) << 16;
            const uint32_t z[16] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
            for (int c = 0; c < (int) cfg::TMEM_COLS; c += 16) tmem_st16(tmem_base + lanes + (uint32_t) c, z);
            tmem_wait_st();
        }
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
    }
    // Test hook: thread 0 waits, with the caller's limit, on the drain barrier
    // before anything has arrived on it. The wait expires; the CTA reports it
    // and skips every role (no copy or MMA has been issued), then frees TMEM.
    bool run = true;
    if (p.stall_ns > 0) {
        if (threadIdx.x == 0) tmem_slot[1] = mbar_wait_for(drain, 0, (uint64_t) p.stall_ns) ? 1u : 0u;
        __syncthreads();
        run = tmem_slot[1] != 0u;
        if (!run && threadIdx.x == 0) atomicExch(p.err, 1);
    }

    if (!run) {
    } else if (warp == 0) {
        if (lane == 0) {
            // ---- TMA producer: counters only, no division per k-step
            uint32_t it = 0;
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            const uint32_t sA0 = smem_u32(sA), sB0 = smem_u32(sB);
            if (BRES) {  // the nine weight taps, once
                // (KHS: slot kw*3 + j holds kernel row 2 - j of column kw, so the
                // three kernel rows of a column are one N = 3 BN operand)
                mbar_expect_tx(bres_bar, cfg::B_RES);
                for (int i = 0; i < 9; i++) {
                    const int tap = KHS ? (2 - i % 3) * 3 + i / 3 : i;
                    tma_load_2d(sB0 + i * cfg::B_TAP, &tmB, bres_bar, tap * p.IC, 0);
                }
            }
            if constexpr (KHS) {  // one halo box per input row of each unit
                for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
                    int b, y0, x0;
                    unit_of(p, t, b, y0, x0);
                    for (int yi = y0 - 1; yi <= y0 + p.yb; yi++) {
                        if (yi < 0 || yi >= p.H) continue;  // zero padding rows: neither load nor MMA
                        if (!mbar_wait(empty(s), ph ^ 1)) {
                            ok = false;
                            break;
                        }
                        mbar_expect_tx(full(s), cfg::STAGE_TX);
                        tma_load_4d(sA0 + s * cfg::A_BYTES, &tmA, full(s), 0, x0 - 1, yi, b);
                        it++;
                        if (++s == cfg::STAGES) {
                            s = 0;
                            ph ^= 1;
                        }
                    }
                }
            } else
            for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
                const tile_pos tp = tile_of(p, t, BN);
                for (int kh = 0; kh < 3 && ok; kh += RPS) {
                    for (int c = 0; c < p.cpt && ok; c++) {
                        for (int kw0 = 0; kw0 < 3; kw0 += cfg::TPS, it++) {
                            // an odd stage was released together with the even one before it
                            if (!(s & 1) && !mbar_wait(empty(s), ph ^ 1)) {
                                ok = false;
                                break;
                            }
                            mbar_expect_tx(full(s), cfg::STAGE_TX);
                            if (HALO)  // pixels x0-1 .. x0+128 of the kernel rows' input rows
#pragma unroll
                                for (int r = 0; r < RPS; r++)
                                    tma_load_4d(sA0 + s * cfg::A_BYTES + r * cfg::A_HALO, &tmA, full(s),
                                                c * KC, tp.x0 - 1, tp.y0 + kh + r - 1, tp.b0);
#pragma unroll
                            for (int i = 0; i < cfg::TPS; i++) {
                                const int kw = kw0 + i;
                                if (!HALO)
                                    tma_load_4d(sA0 + s * cfg::A_BYTES + i * cfg::A_TAP, &tmA, full(s),
                                                c * KC, tp.x0 + kw - 1, tp.y0 + kh - 1, tp.b0);
                                // weight column of (tap, chunk): tap * IC + c * KC
                                if (!BRES)
                                    tma_load_2d(sB0 + s * cfg::B_BYTES + i * cfg::B_TAP, &tmB, full(s),
                                                (kh * 3 + kw) * p.IC + c * KC, tp.n0);
                            }
                            if (++s == cfg::STAGES) {
                                s = 0;
                                ph ^= 1;
                            }
                        }
                    }
                }
            }
            if (!ok) {
                atomicExch(p.err, 1);
                // let the loads already issued land before shared memory goes away
                for (int s = 0; s < cfg::STAGES && (uint32_t) s < it; s++) {
                    const uint32_t last = it - 1 - ((it - 1 - s) % cfg::STAGES);
                    mbar_wait(full(s), (last / cfg::STAGES) & 1);
                }
                if (BRES) mbar_wait(bres_bar, 0);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer: tile k of this CTA accumulates into buffer k % NACC
            int s = 0, a = 0;
            uint32_t ph = 0, aph = 0;
            bool ok = true;
            // descriptors of stage 0; stage s adds its byte offset >> 4 to the
            // start-address field (shared addresses stay below 2^18)
            const uint64_t ad0 = smem_desc(smem_u32(sA), cfg::SBO, cfg::LAYOUT);
            const uint64_t bd0 = smem_desc(smem_u32(sB), cfg::SBO, cfg::LAYOUT);
            if (BRES && !mbar_wait(bres_bar, 0)) ok = false;
            if constexpr (KHS) {
                // output row rc of this CTA (counted over its units) accumulates
                // in slot rc % R, its (rc / R)-th use
                uint32_t rc0 = 0;
                for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
                    int b, y0, x0;
                    unit_of(p, t, b, y0, x0);
                    const int yend = y0 + p.yb;
                    for (int yi = y0 - 1; yi <= yend; yi++) {
                        if (yi + 1 < yend) {  // row yi + 1 is first touched here: its slot must be free
                            const uint32_t rc = rc0 + (uint32_t) (yi + 1 - y0);
                            if (rc >= (uint32_t) cfg::R &&
                                !mbar_wait(tempty(rc % cfg::R), ((rc / cfg::R) - 1) & 1)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();  // the epilogue's clearing stores come first
                        }
                        if (yi >= 0 && yi < p.H) {
                            if (!mbar_wait(full(s), ph)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            // blocks j = jlo..jhi: the output rows yi - 1 + j of this strip,
                            // in consecutive slots except where the ring wraps
                            const int jlo = max(0, y0 - (yi - 1)), jhi = min(2, yend - yi);
                            const int nb = jhi - jlo + 1;
                            const uint32_t sl = (rc0 + (uint32_t) (yi - 1 + jlo - y0)) % cfg::R;
                            const int n1 = min(nb, cfg::R - (int) sl);
                            const uint64_t ad = ad0 + (uint64_t) ((s * cfg::A_BYTES) >> 4);
#pragma unroll
                            for (int kw = 0; kw < 3; kw++)
#pragma unroll
                                for (int kx = 0; kx < KC / 16; kx++) {  // +32 bytes along K per step
                                    const uint64_t a_d = ad + ((kw * KC * 2) >> 4) + 2 * kx;
                                    const uint64_t b_d = bd0 + (((kw * 3 + jlo) * cfg::B_TAP) >> 4) + 2 * kx;
                                    umma_f16(tmem_base + sl * BN, a_d, b_d, cfg::idesc_n(n1), 1);
                                    if (n1 < nb)
                                        umma_f16(tmem_base, a_d, b_d + ((n1 * cfg::B_TAP) >> 4), cfg::idesc_n(nb - n1), 1);
                                }
                            umma_commit(empty(s));
                            if (++s == cfg::STAGES) {
                                s = 0;
                                ph ^= 1;
                            }
                        }
                        if (yi - 1 >= y0)  // output row yi - 1 has all its contributions
                            umma_commit(tfull((rc0 + (uint32_t) (yi - 1 - y0)) % cfg::R));
                    }
                    rc0 += (uint32_t) p.yb;
                }
            } else
            for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
                if (!mbar_wait(tempty(a), aph ^ 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + a * BN;
                int tap0 = 0;  // first tap of the stage (BRES: its resident B tile)
                for (int kk = 0; kk < p.kiters; kk++, tap0 += cfg::TAPS) {
                    if (!mbar_wait(full(s), ph)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t ad = ad0 + (uint64_t) ((s * cfg::A_BYTES) >> 4);
                    const uint64_t bd = BRES ? bd0 + (uint64_t) ((tap0 * cfg::B_TAP) >> 4)
                                             : bd0 + (uint64_t) ((s * cfg::B_BYTES) >> 4);
#pragma unroll
                    for (int i = 0; i < cfg::TAPS; i++)
#pragma unroll
                        for (int kx = 0; kx < KC / 16; kx++)  // +32 bytes along K per step
                            umma_f16(d_tmem,
                                     ad + (((HALO ? (i / 3) * cfg::A_HALO + (i % 3) * KC * 2 : i * cfg::A_TAP)) >> 4) +
                                         2 * kx,
                                     bd + ((i * cfg::B_TAP) >> 4) + 2 * kx, cfg::IDESC, (kk | i | kx) != 0);
                    if (s & 1) umma_commit(empty(s));  // releases stages s-1 and s
                    if (++s == cfg::STAGES) {
                        s = 0;
                        ph ^= 1;
                    }
                }
                if (!ok) break;
                umma_commit(tfull(a));
                if (++a == NACC) {
                    a = 0;
                    aph ^= 1;
                }
            }
            if (!ok) atomicExch(p.err, 1);
            umma_commit(drain);  // completes when every MMA issued here has
            mbar_wait(drain, 0);
        }
    } else {
        // ---- epilogue group g = (warp-2)/4 owns accumulator g and the CTA's
        // tiles k = g, g+NACC, ...; each warp reads TMEM lane quarter warp % 4
        const int g = (warp - 2) >> 2;
        const int q = warp & 3;
        const int row = q * 32 + lane;
        const int bx = row % p.bw, by = (row / p.bw) % p.bh, bz = row / (p.bw * p.bh);
        const uint32_t lanes = (uint32_t) (q * 32) << 16;
        const float *s_fw = sx, *s_up = sx + 3 * BN;
        float *s_cst = sx + 3 * BN + 32 + g * 2 * cfg::CW;  // this group's two constant buffers
        // this warp's trunk exchange area (XCH)
        float *s_xw = sx + 3 * BN + 32 + (cfg::STG ? NACC * 2 * cfg::CW : 0) + (warp - 2) * cfg::XW;
        uint32_t nst = 0;  // stagings this group has made
        int cur_b = -1;    // the frame whose constants are staged
        // one tile's epilogue: its accumulator at taddr0 is complete once
        // barrier `bar` finishes phase `par`; false if that wait timed out
        auto tile_body = [&](const tile_pos &tp, uint32_t taddr0, uint32_t bar, uint32_t par) -> bool {
            const int b = tp.b0 + bz, y = tp.y0 + by, x = tp.x0 + bx;
            // TAIL: the up-sampled flow and rgb skips depend on the pixel only;
            // their loads are issued before the wait for the accumulator
            float skf[3] = {0.0f, 0.0f, 0.0f}, skr[3] = {0.0f, 0.0f, 0.0f};
            if constexpr (TAIL) {
                const int h = p.W >> 1;
                const int px = x & 1, py = y & 1, nx = x >> 1, ny = y >> 1;
                int uoff[4];
                float ukf[4], ukr[4];
#pragma unroll
                for (int a = 0; a < 2; a++)
#pragma unroll
                    for (int bb = 0; bb < 2; bb++) {
                        const int sy = ny + py - 1 + a, sx2 = nx + px - 1 + bb;
                        const bool in = sy >= 0 && sy < h && sx2 >= 0 && sx2 < h;
                        const int uk = (px + 2 * bb) + 4 * (py + 2 * a);
                        // taps outside the map read pixel 0 with weight 0 (no branches)
                        uoff[2 * a + bb] = in ? sy * h + sx2 : 0;
                        ukf[2 * a + bb] = in ? s_up[uk] : 0.0f;
                        ukr[2 * a + bb] = in ? s_up[16 + uk] : 0.0f;
                    }
                const int64_t hh = (int64_t) h * h;
                if (p.skipf_prev) {
#pragma unroll
                    for (int kk = 0; kk < 3; kk++) {
                        const float *pl = p.skipf_prev + ((int64_t) b * 3 + kk) * hh;
#pragma unroll
                        for (int i = 0; i < 4; i++)
                            skf[kk] = fmaf(__ldg(pl + uoff[i]), ukf[i], skf[kk]);
                    }
                }
                if (p.skip_prev) {
#pragma unroll
                    for (int kk = 0; kk < 3; kk++) {
                        const float *pl = p.skip_prev + ((int64_t) b * 3 + kk) * hh;
#pragma unroll
                        for (int i = 0; i < 4; i++)
                            skr[kk] = fmaf(__ldg(pl + uoff[i]), ukr[i], skr[kk]);
                    }
                }
            }
            // STG: stage the frame's channel constants when the group's frame
            // changes: the group's 128 threads write, arrive on the group's
            // barrier and wait (bounded) for its phase. The two buffers
            // alternate, so a buffer is rewritten only after every thread of
            // the group has completed the phase of the staging after the one
            // that filled it (reached only after all tiles that read it)
            if constexpr (cfg::STG) {
                if (b != cur_b) {
                float *cst = s_cst + (nst & 1) * cfg::CW;
                const float *fden = p.inv_den + (int64_t) b * p.den_stride;
                const float *ffs = p.fs + (int64_t) b * p.s_stride;
                for (int c = row; c < BN; c += 128) {
                    const float fsv = __ldg(ffs + c);
                    cst[c] = __ldg(fden + c);
                    cst[BN + c] = __ldg(p.bias + c);
                    cst[2 * BN + c] = s_fw[c] * fsv;
                    cst[3 * BN + c] = s_fw[BN + c] * fsv;
                    cst[4 * BN + c] = s_fw[2 * BN + c] * fsv;
                    if (p.trunk) cst[5 * BN + c] = __ldg(p.tsn + (int64_t) b * p.s_stride + c);
                }
                mbar_arrive(cbar(g));
                if (!__all_sync(0xffffffffu, mbar_wait(cbar(g), nst & 1))) {
                    if (lane == 0) atomicExch(p.err, 1);
                    return false;
                }
                nst++;
                cur_b = b;
                }
            }
            const float *cst = s_cst + ((nst - 1) & 1) * cfg::CW;
            const bool ok = __all_sync(0xffffffffu, mbar_wait(bar, par));
            if (!ok) {
                if (lane == 0) atomicExch(p.err, 1);
                return false;
            }
            tc_fence_after();
            if constexpr (!TAIL) {
                const bool valid = b < p.B;
                // the tile's columns are ncls sub-pixel classes (UP) of `span`
                // channels each, column = class * OC + channel; a channel's
                // per-frame constants are loaded once for all its classes
                const int span = UP ? (BN < p.OC ? BN : p.OC) : BN;
                const int ncls = BN / span;
                const int cls0 = UP ? tp.n0 >> p.lg_oc : 0;
                const int obase = UP ? tp.n0 & (p.OC - 1) : tp.n0;
#pragma unroll 1
                for (int c0 = 0; c0 < span; c0 += 16) {
                    const int o0 = obase + c0;
                    float den[16], bias[16], sn[16];
                    if (valid) {
                        const float4 *dp =
                            reinterpret_cast<const float4 *>(p.inv_den + (int64_t) b * p.den_stride + o0);
                        const float4 *bp = reinterpret_cast<const float4 *>(p.bias + o0);
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            const float4 dv = __ldg(dp + i), bv = __ldg(bp + i);
                            den[4 * i] = dv.x; den[4 * i + 1] = dv.y; den[4 * i + 2] = dv.z; den[4 * i + 3] = dv.w;
                            bias[4 * i] = bv.x; bias[4 * i + 1] = bv.y; bias[4 * i + 2] = bv.z; bias[4 * i + 3] = bv.w;
                        }
                        if (p.snext) {
                            const float4 *sp =
                                reinterpret_cast<const float4 *>(p.snext + (int64_t) b * p.snext_stride + o0);
#pragma unroll
                            for (int i = 0; i < 4; i++) {
                                const float4 sv = __ldg(sp + i);
                                sn[4 * i] = sv.x; sn[4 * i + 1] = sv.y; sn[4 * i + 2] = sv.z; sn[4 * i + 3] = sv.w;
                            }
                        }
                    }
#pragma unroll 1
                    for (int k = 0; k < ncls; k++) {
                        uint32_t r[16];
                        tmem_ld16(taddr0 + k * span + c0, r);
                        if (!valid) continue;
                        float v[16];
#pragma unroll
                        for (int i = 0; i < 16; i++) {
                            float a = fmaf(__uint_as_float(r[i]), den[i], bias[i]);
                            a = fmaxf(a, 0.2f * a);  // leaky relu, slope 0.2
                            v[i] = p.snext ? a * sn[i] : a;
                        }
                        int64_t dst;
                        if (UP) {
                            const int cls = cls0 + k;
                            const int Y = 2 * y + (cls >> 1), X = 2 * x + (cls & 1);
                            dst = (((int64_t) b * 2 * p.H + Y) * 2 * p.W + X) * p.OC + o0;
                        } else {
                            dst = (((int64_t) b * p.H + y) * p.W + x) * p.OC + o0;
                        }
                        st_half16(p.y + dst, v);
                    }
                }
            } else {
                // ---- conv2 + level tail (one tile = 128 pixels of one frame,
                // BN = OC: every channel of a pixel is in this thread's TMEM lane)
                const float *fden = p.inv_den + (int64_t) b * p.den_stride;
                const float *ffs = p.fs + (int64_t) b * p.s_stride;
                const float *fsn = p.trunk ? p.tsn + (int64_t) b * p.s_stride : nullptr;
                const float4 *c_den = reinterpret_cast<const float4 *>(cst);
                const float4 *c_bias = reinterpret_cast<const float4 *>(cst + BN);
                const float4 *c_g0 = reinterpret_cast<const float4 *>(cst + 2 * BN);
                const float4 *c_g1 = reinterpret_cast<const float4 *>(cst + 3 * BN);
                const float4 *c_g2 = reinterpret_cast<const float4 *>(cst + 4 * BN);
                const float4 *c_sn = reinterpret_cast<const float4 *>(cst + 5 * BN);
                const int r = p.W;
                const int64_t pix = ((int64_t) b * p.H + y) * p.W + x;
                // the last level has no trunk: it needs neither the conv2 output
                // nor TMEM after pass 1
                const bool need_out = p.trunk != nullptr;
                // pass 1: conv2 output (f32, never stored) -> ToFlow sums; the
                // activation goes back into TMEM for pass 2
                float f0 = 0.0f, f1 = 0.0f, f2 = 0.0f;
#pragma unroll 1
                for (int c0 = 0; c0 < BN; c0 += 16) {
                    uint32_t rr[16];
                    tmem_ld16(taddr0 + c0, rr);
                    float v[16];
                    if constexpr (!cfg::STG) {
                        float den[16], bias[16], fsv[16];
                        ld_f16x(fden + c0, den);
                        ld_f16x(p.bias + c0, bias);
                        ld_f16x(ffs + c0, fsv);
#pragma unroll
                        for (int i = 0; i < 16; i++) {
                            float a = fmaf(__uint_as_float(rr[i]), den[i], bias[i]);
                            a = fmaxf(a, 0.2f * a);  // leaky relu, slope 0.2
                            v[i] = a;
                            rr[i] = __float_as_uint(a);
                            const float xs = a * fsv[i];  // ToFlow input: out * style
                            f0 = fmaf(s_fw[c0 + i], xs, f0);
                            f1 = fmaf(s_fw[BN + c0 + i], xs, f1);
                            f2 = fmaf(s_fw[2 * BN + c0 + i], xs, f2);
                        }
                    } else {
#pragma unroll
                    for (int i4 = 0; i4 < 4; i4++) {
                        // four channels' constants: five broadcast 16-byte shared loads
                        const int q4 = (c0 >> 2) + i4;
                        const float4 dn = c_den[q4], bs = c_bias[q4], w0 = c_g0[q4], w1 = c_g1[q4],
                                     w2 = c_g2[q4];
                        const float dnv[4] = {dn.x, dn.y, dn.z, dn.w}, bsv[4] = {bs.x, bs.y, bs.z, bs.w};
                        const float w0v[4] = {w0.x, w0.y, w0.z, w0.w}, w1v[4] = {w1.x, w1.y, w1.z, w1.w};
                        const float w2v[4] = {w2.x, w2.y, w2.z, w2.w};
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            const int i = 4 * i4 + j;
                            float a = fmaf(__uint_as_float(rr[i]), dnv[j], bsv[j]);
                            a = fmaxf(a, 0.2f * a);  // leaky relu, slope 0.2
                            v[i] = a;
                            rr[i] = __float_as_uint(a);
                            // ToFlow of out * style: the style is folded into the weights
                            f0 = fmaf(w0v[j], a, f0);
                            f1 = fmaf(w1v[j], a, f1);
                            f2 = fmaf(w2v[j], a, f2);
                        }
                    }
                    }
                    if (need_out) tmem_st16(taddr0 + c0, rr);
                    if (p.y) st_half16(p.y + pix * BN + c0, v);  // conv2 tap (debug)
                }
                if (need_out) tmem_wait_st();
                float fl[3] = {f0 + __ldg(p.fb), f1 + __ldg(p.fb + 1), f2 + __ldg(p.fb + 2)};
#pragma unroll
                for (int kk = 0; kk < 3; kk++) fl[kk] += skf[kk];
                const int64_t rr2 = (int64_t) r * r;
                if (p.skipf_out) {
#pragma unroll
                    for (int kk = 0; kk < 3; kk++) p.skipf_out[((int64_t) b * 3 + kk) * rr2 + (int64_t) y * r + x] = fl[kk];
                }
                const float gx = tanhf(fl[0]) + __ldg(p.lin + x);
                const float gy = tanhf(fl[1]) + __ldg(p.lin + y);
                const float m = 1.0f / (1.0f + expf(-fl[2]));
                const float om = 1.0f - m;
                // bilinear taps, as the patched gather computes them (patch:341-358)
                const float fx = fmaf((gx + 1.0f) * 0.5f, (float) r, -0.5f);
                const float fy = fmaf((gy + 1.0f) * 0.5f, (float) r, -0.5f);
                const bool sane = fabsf(fx) < 1.0e8f && fabsf(fy) < 1.0e8f;
                const float flx = floorf(fx), fly = floorf(fy);
                const int x0 = sane ? (int) flx : -4, y0 = sane ? (int) fly : -4;
                const float wx = fx - flx, wy = fy - fly;
                int trow[4];
                float twt[4];
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                    const int cx = x0 + (kk & 1), cy = y0 + (kk >> 1);
                    // a tap outside the map (zeros padding) reads pixel 0 with weight 0
                    const bool in = sane && cx >= 0 && cx < r && cy >= 0 && cy < r;
                    trow[kk] = in ? cy * r + cx : 0;
                    twt[kk] = in ? ((kk & 1) ? wx : 1.0f - wx) * ((kk >> 1) ? wy : 1.0f - wy) : 0.0f;
                }
                // ToRGB of the gathered channels = gather of the feats projected
                // by ToRGB's 1x1 conv (both linear): four 16-byte taps
                float g0 = 0.0f, g1 = 0.0f, g2 = 0.0f;
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                    const float4 pq = __ldg(p.proj + trow[kk]);
                    g0 = fmaf(twt[kk], pq.x, g0);
                    g1 = fmaf(twt[kk], pq.y, g1);
                    g2 = fmaf(twt[kk], pq.z, g2);
                }
                // pass 2 (levels with a trunk): gather, blend, trunk. Per 32-channel
                // slice, four rounds of eight pixels: the eight owners publish their
                // activations (f32, from TMEM) and tap geometry in the warp's exchange
                // area; then four lanes per pixel each gather, blend and store eight
                // channels, so a warp's feats loads and trunk stores cover eight
                // 64-byte runs instead of 32 scattered 16-byte pieces
                if constexpr (cfg::XCH) {
                    float *xa = s_xw;                                    // [8][36]
                    int *xm = reinterpret_cast<int *>(s_xw + 8 * 36);    // [8][12]
                    const int pg = lane >> 2, sub = lane & 3;
#pragma unroll 1
                    for (int s0 = 0; s0 < BN && need_out; s0 += 32) {
#pragma unroll 1
                        for (int it = 0; it < 4; it++) {
                            // the slice is re-read from TMEM each round (a warp-wide
                            // load; only this round's owners keep it), which holds
                            // fewer registers live than keeping it across rounds
                            uint32_t a0[16], a1[16];
                            tmem_ld16(taddr0 + s0, a0);
                            tmem_ld16(taddr0 + s0 + 16, a1);
                            if ((lane >> 3) == it) {
                                float4 *d4 = reinterpret_cast<float4 *>(xa + (lane & 7) * 36);
#pragma unroll
                                for (int j = 0; j < 4; j++) {
                                    d4[j] = make_float4(__uint_as_float(a0[4 * j]), __uint_as_float(a0[4 * j + 1]),
                                                        __uint_as_float(a0[4 * j + 2]), __uint_as_float(a0[4 * j + 3]));
                                    d4[4 + j] = make_float4(__uint_as_float(a1[4 * j]), __uint_as_float(a1[4 * j + 1]),
                                                            __uint_as_float(a1[4 * j + 2]), __uint_as_float(a1[4 * j + 3]));
                                }
                                int4 *m4 = reinterpret_cast<int4 *>(xm + (lane & 7) * 12);
                                m4[0] = make_int4(trow[0], trow[1], trow[2], trow[3]);
                                m4[1] = make_int4(__float_as_int(twt[0]), __float_as_int(twt[1]),
                                                  __float_as_int(twt[2]), __float_as_int(twt[3]));
                                m4[2] = make_int4(__float_as_int(m), (int) (uint32_t) pix, (int) (pix >> 32), 0);
                            }
                            __syncwarp();
                            const int4 *m4 = reinterpret_cast<const int4 *>(xm + pg * 12);
                            const int4 tr = m4[0], tw = m4[1], mp = m4[2];
                            const int trk[4] = {tr.x, tr.y, tr.z, tr.w};
                            const float twk[4] = {__int_as_float(tw.x), __int_as_float(tw.y), __int_as_float(tw.z),
                                                  __int_as_float(tw.w)};
                            const float mq = __int_as_float(mp.x), omq = 1.0f - mq;
                            const int64_t pq = (int64_t) (((uint64_t) (uint32_t) mp.z << 32) | (uint32_t) mp.y);
                            const int cc = s0 + sub * 8;
                            float smp[8];
#pragma unroll
                            for (int i = 0; i < 8; i++) smp[i] = 0.0f;
#pragma unroll
                            for (int kk = 0; kk < 4; kk++) {
                                float f[8];
                                ld_half8(p.feat + (int64_t) trk[kk] * BN + cc, f);
#pragma unroll
                                for (int i = 0; i < 8; i++) smp[i] = fmaf(twk[kk], f[i], smp[i]);
                            }
                            const float4 *ar = reinterpret_cast<const float4 *>(xa + pg * 36 + sub * 8);
                            const float4 av0 = ar[0], av1 = ar[1];
                            const float av[8] = {av0.x, av0.y, av0.z, av0.w, av1.x, av1.y, av1.z, av1.w};
                            float4 sv0, sv1;
                            if constexpr (cfg::STG) {
                                sv0 = c_sn[cc >> 2];
                                sv1 = c_sn[(cc >> 2) + 1];
                            } else {
                                sv0 = __ldg(reinterpret_cast<const float4 *>(fsn + cc));
                                sv1 = __ldg(reinterpret_cast<const float4 *>(fsn + cc) + 1);
                            }
                            const float sn[8] = {sv0.x, sv0.y, sv0.z, sv0.w, sv1.x, sv1.y, sv1.z, sv1.w};
                            float o[8];
#pragma unroll
                            for (int i = 0; i < 8; i++) {
                                const float w = smp[i] * mq;
                                o[i] = (w + av[i] * omq) * sn[i];  // trunk x next up-conv style
                            }
                            st_half8(p.trunk + pq * BN + cc, o);
                            __syncwarp();
                        }
                    }
                } else {
#pragma unroll 1
                for (int c0 = 0; c0 < BN && need_out; c0 += 16) {
                    uint32_t rr[16];
                    tmem_ld16(taddr0 + c0, rr);
                    float smp[16];
#pragma unroll
                    for (int i = 0; i < 16; i++) smp[i] = 0.0f;
#pragma unroll
                    for (int kk = 0; kk < 4; kk++) {
                        float f[16];
                        ld_half16(p.feat + (int64_t) trow[kk] * BN + c0, f);
#pragma unroll
                        for (int i = 0; i < 16; i++) smp[i] = fmaf(twt[kk], f[i], smp[i]);
                    }
                    float sn[16];
                    if constexpr (!cfg::STG) {
                        ld_f16x(fsn + c0, sn);
                    } else {
#pragma unroll
                        for (int i4 = 0; i4 < 4; i4++) {
                            const float4 t = c_sn[(c0 >> 2) + i4];
                            sn[4 * i4] = t.x;
                            sn[4 * i4 + 1] = t.y;
                            sn[4 * i4 + 2] = t.z;
                            sn[4 * i4 + 3] = t.w;
                        }
                    }
#pragma unroll
                    for (int i = 0; i < 16; i++) {
                        const float w = smp[i] * m;
                        smp[i] = (w + __uint_as_float(rr[i]) * om) * sn[i];  // trunk x next up-conv style
                    }
                    st_half16(p.trunk + pix * BN + c0, smp);
                }
                }
                const float rg[3] = {g0 * m, g1 * m, g2 * m};
#pragma unroll
                for (int kk = 0; kk < 3; kk++) {
                    float v = rg[kk] + __ldg(p.rlb + kk);
                    v = fmaxf(v, 0.2f * v) + __ldg(p.rb + kk);
                    if (p.skip_prev) v += skr[kk];
                    p.skip_out[((int64_t) b * 3 + kk) * rr2 + (int64_t) y * r + x] = v;
                }
            }
            return true;
        };
        if constexpr (KHS) {
            // group g takes the output rows rc = g, g + NACC, ... of the CTA's units
            // (p.yb is a multiple of NACC); after each row it clears the row's slot
            const uint32_t z[16] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
            uint32_t rc0 = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
                tile_pos tp;
                tp.n0 = 0;
                unit_of(p, t, tp.b0, tp.y0, tp.x0);
                const int y0 = tp.y0;
                for (int i = g; i < p.yb; i += NACC) {
                    const uint32_t rc = rc0 + (uint32_t) i, sl = rc % cfg::R;
                    const uint32_t slot = tmem_base + lanes + sl * BN;
                    tp.y0 = y0 + i;
                    if (!tile_body(tp, slot, tfull(sl), (rc / cfg::R) & 1)) {
                        ok = false;
                        break;
                    }
#pragma unroll
                    for (int c0 = 0; c0 < BN; c0 += 16) tmem_st16(slot + c0, z);
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(tempty(sl));
                }
                rc0 += (uint32_t) p.yb;
            }
        } else {
            uint32_t k = g;
            for (int t = blockIdx.x + g * gridDim.x; t < p.num_tiles; t += NACC * gridDim.x, k += NACC) {
                if (!tile_body(tile_of(p, t, BN), tmem_base + lanes + g * BN, tfull(g), (k / NACC) & 1)) break;
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(tempty(g));
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                     "r"(cfg::TMEM_COLS)
                     : "memory");
}

// ---- host side ------------------------------------------------------------
int ilog2(int v) {  // log2 of a power of two, else -1
    if (v <= 0 || (v & (v - 1))) return -1;
    int l = 0;
    while ((1 << l) < v) l++;
    return l;
}


template <int BN, int KC, bool UP, int NACC, bool TAIL, bool BRES = false, bool HALO = false, int RPS = 1,
          bool KHS = false, bool DEEP = false>
cudaError_t run_tc(const conv_params &cp, const tail_params *tl, cudaStream_t st) {
    using cfg = tc_cfg<BN, KC, NACC, TAIL, BRES, HALO, RPS, KHS, DEEP>;
    auto enc = encode_fn();
    if (!enc) return cudaErrorNotSupported;
    tc_params p{};
    p.B = cp.B;
    p.H = cp.H;
    p.W = cp.W;
    p.IC = cp.IC;
    p.OC = cp.OC;
    p.N = UP ? 4 * cp.OC : cp.OC;
    p.cpt = cp.IC / KC;
    p.kiters = 9 * p.cpt / cfg::TAPS;  // pipeline stages per tile
    p.bw = cp.W < BM ? cp.W : BM;
    p.bh = cp.H < BM / p.bw ? cp.H : BM / p.bw;
    p.bb = BM / (p.bw * p.bh);
    p.tiles_x = cp.W / p.bw;
    p.tiles_y = cp.H / p.bh;
    p.tiles_n = p.N / BN;
    p.lg_x = ilog2(p.tiles_x);
    p.lg_y = ilog2(p.tiles_y);
    p.lg_n = ilog2(p.tiles_n);
    p.lg_oc = ilog2(cp.OC);
    if (p.lg_x < 0 || p.lg_y < 0 || p.lg_n < 0 || p.lg_oc < 0 || p.N % BN) return cudaErrorInvalidValue;
    if (UP && (BN % 16 || (BN > cp.OC && BN % cp.OC))) return cudaErrorInvalidValue;
    const int tiles_b = (cp.B + p.bb - 1) / p.bb;
    int64_t nt = (int64_t) tiles_b * p.tiles_y * p.tiles_x * p.tiles_n;
    if (KHS) {
        // units of yb output rows: the longest strips that still give every SM
        // at least 8 units (the row count per CTA then differs by a few percent)
        if (p.bw != BM || cp.W % BM || cp.H % 8) return cudaErrorInvalidValue;
        p.yb = 8;
        for (int c = 32; c > 8; c >>= 1)
            if (cp.H % c == 0 && (int64_t) cp.B * (cp.H / c) * p.tiles_x >= 8 * sm_count()) {
                p.yb = c;
                break;
            }
        p.strips = cp.H / p.yb;
        nt = (int64_t) cp.B * p.strips * p.tiles_x;
    }
    if (nt >= (1ll << 30)) return cudaErrorInvalidValue;
    p.num_tiles = (int) nt;
    if (BRES && (p.cpt != 1 || p.tiles_n != 1)) return cudaErrorInvalidValue;  // 9 taps x 1 chunk, 1 N tile
    if (HALO && (p.bw != BM || p.bh != 1 || p.bb != 1)) return cudaErrorInvalidValue;  // one-row tiles
    p.y = (__half *) cp.y;
    p.inv_den = cp.inv_den;
    p.den_stride = cp.den_stride;
    p.bias = cp.bias;
    p.snext = cp.snext;
    p.snext_stride = cp.snext_stride;
    p.err = cp.err;
    p.stall_ns = cp.stall_ns;
    if (TAIL) {
        // one frame per tile and the whole channel range in one tile
        if (!tl || !tl->proj || p.bb != 1 || p.tiles_n != 1 || tl->OC != BN || tl->r != cp.W)
            return cudaErrorInvalidValue;
        p.feat = (const __half *) tl->feat;
        p.fW = tl->fW;
        p.fs = tl->fs;
        p.s_stride = tl->s_stride;
        p.fb = tl->fb;
        p.fup = tl->fup;
        p.skipf_prev = tl->skipf_prev;
        p.skipf_out = tl->skipf_out;
        p.rW = tl->rW;
        p.rlb = tl->rlb;
        p.rb = tl->rb;
        p.rup = tl->rup;
        p.skip_prev = tl->skip_prev;
        p.skip_out = tl->skip_out;
        p.lin = tl->lin;
        p.trunk = (__half *) tl->trunk;
        p.tsn = tl->snext;
        p.proj = tl->proj;
    }

    CUtensorMap tmA, tmB;
    {
        const cuuint64_t dims[4] = {(cuuint64_t) cp.IC, (cuuint64_t) cp.W, (cuuint64_t) cp.H,
                                    (cuuint64_t) cp.B};
        const cuuint64_t strides[3] = {(cuuint64_t) cp.IC * 2, (cuuint64_t) cp.W * cp.IC * 2,
                                       (cuuint64_t) cp.H * cp.W * cp.IC * 2};
        const cuuint32_t box[4] = {(cuuint32_t) KC, (cuuint32_t) (HALO ? cfg::HALO_ROWS : p.bw),
                                   (cuuint32_t) p.bh, (cuuint32_t) p.bb};
        const cuuint32_t es[4] = {1, 1, 1, 1};
        if (enc(&tmA, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, (void *) cp.x, dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE,
                KC == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    {
        const int K = 9 * cp.IC;
        const cuuint64_t dims[2] = {(cuuint64_t) K, (cuuint64_t) p.N};
        const cuuint64_t strides[1] = {(cuuint64_t) K * 2};
        const cuuint32_t box[2] = {(cuuint32_t) KC, (cuuint32_t) BN};
        const cuuint32_t es[2] = {1, 1};
        if (enc(&tmB, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void *) cp.w, dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE,
                KC == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    static uint64_t attr_set = 0;  // one bit per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(attr_set >> (dev & 63) & 1)) {
        const cudaError_t e = cudaFuncSetAttribute(conv_tc_kernel<BN, KC, UP, NACC, TAIL, BRES, HALO, RPS, KHS, DEEP>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize, cfg::SMEM);
        if (e != cudaSuccess) return e;
        attr_set |= 1ull << (dev & 63);
    }
    const int grid = (int) (p.num_tiles < sm_count() ? p.num_tiles : sm_count());
    conv_tc_kernel<BN, KC, UP, NACC, TAIL, BRES, HALO, RPS, KHS, DEEP><<<grid, cfg::THREADS, cfg::SMEM, st>>>(tmA, tmB, p);
    return cudaGetLastError();
}

}  // namespace

bool conv_tc_supported(bool up, int IC, int OC) {
    const int N = up ? 4 * OC : OC;
    if (IC % 32 != 0 || OC % 16 != 0) return false;
    if (IC == 32) return !up && N == 32;
    return IC % 64 == 0 && (N >= 256 ? N % 256 == 0 : (N == 128 || N == 64));
}

cudaError_t launch_conv_tc(bool up, const conv_params &p, cudaStream_t st) {
    const int N = up ? 4 * p.OC : p.OC;
    if (!conv_tc_supported(up, p.IC, p.OC) || !p.err) return cudaErrorInvalidValue;
    if (p.IC == 32) return run_tc<32, 32, false, 4, false>(p, nullptr, st);
    // 128-pixel M tiles, as run_tc forms them
    const int bw = p.W < BM ? p.W : BM, bh = p.H < BM / bw ? p.H : BM / bw, bb = BM / (bw * bh);
    const int64_t m_tiles = (int64_t) ((p.B + bb - 1) / bb) * (p.H / bh) * (p.W / bw);
    // the small early levels (4x4 .. 8x8 maps) leave most SMs idle with
    // 256-wide N tiles; 128-wide ones double the tile count at the same K
    if (N >= 256 && m_tiles * (N / 256) < sm_count()) {
        // and with fewer 128-wide tiles than SMs, one tap per stage (DEEP)
        if (m_tiles * (N / 128) < sm_count())
            return up ? run_tc<128, 64, true, 4, false, false, false, 1, false, true>(p, nullptr, st)
                      : run_tc<128, 64, false, 4, false, false, false, 1, false, true>(p, nullptr, st);
        return up ? run_tc<128, 64, true, 4, false>(p, nullptr, st)
                  : run_tc<128, 64, false, 4, false>(p, nullptr, st);
    }
    if (N >= 256)
        return up ? run_tc<256, 64, true, 2, false>(p, nullptr, st)
                  : run_tc<256, 64, false, 2, false>(p, nullptr, st);
    if (N == 128 && up && p.IC == 64) {
        if (p.W >= BM) return run_tc<128, 64, true, 4, false, true, true>(p, nullptr, st);
        return run_tc<128, 64, true, 4, false, true>(p, nullptr, st);
    }
    if (N == 128)
        return up ? run_tc<128, 64, true, 4, false>(p, nullptr, st)
                  : run_tc<128, 64, false, 4, false>(p, nullptr, st);
    return up ? run_tc<64, 64, true, 4, false>(p, nullptr, st) : run_tc<64, 64, false, 4, false>(p, nullptr, st);
}

bool conv_tail_tc_supported(int IC, int OC, int r) {
    // OC = 128 runs with one-row halo tiles only (maps >= 128 wide, the r128
    // level): a 128-wide non-halo tile leaves no room for two stages next to
    // the staged per-frame constants
    return IC == OC && (OC == 32 || OC == 64 || OC == 128 || OC == 256) && r >= (OC == 128 ? 128 : 64);
}

cudaError_t launch_conv_tail_tc(const conv_params &p, const tail_params &t, cudaStream_t st) {
    if (!conv_tail_tc_supported(p.IC, p.OC, p.W) || !p.err || p.H != p.W) return cudaErrorInvalidValue;
    const bool halo = p.W >= BM;  // one-row tiles: taps share a halo box
    switch (p.OC) {
        case 32:  // halo: kernel rows stacked in N, row accumulators in a TMEM ring
            return halo ? run_tc<32, 32, false, 4, true, true, true, 1, true>(p, &t, st)
                        : run_tc<32, 32, false, 4, true, true>(p, &t, st);
        case 64:  // (stacked kernel rows measured slower here: 6 one-row stages)
            return halo ? run_tc<64, 64, false, 4, true, true, true, 3>(p, &t, st)
                        : run_tc<64, 64, false, 4, true>(p, &t, st);
        case 128:
            return halo ? run_tc<128, 64, false, 4, true, false, true>(p, &t, st) : cudaErrorInvalidValue;
        default: return run_tc<256, 64, false, 2, true>(p, &t, st);
    }
}

}  // namespace tpmd
