// C++ shim over tpmd.h with the method shape the reference's pipeline uses
// for its decoder (tp::motion_dec, src/motion_dec.h:10-49; called from
// src/pipeline.cpp:153-184): build / set_feats / decode_batch / batch /
// built / taps_in_graph, errors as bool + std::string. Header-only; link
// libtpmd.so.
#pragma once

#include <cstring>
#include <string>
#include <vector>

#include "tpmd.h"

namespace tpmd_cpp {

struct motion_dec_b200 {
    tpmd_ctx *ctx = nullptr;
    bool built = false;
    bool taps_in_graph = false;  // the tap plan is tpmd_decode_taps, never the decode plan
    int batch = 8;               // frames per decode_batch call (the reference's BQ)

    motion_dec_b200() = default;
    motion_dec_b200(const motion_dec_b200 &) = delete;
    motion_dec_b200 &operator=(const motion_dec_b200 &) = delete;
    ~motion_dec_b200() { release(); }

    // tp_ctx::load's decoder half (src/tp.cpp:32-39): device, "f32"/"f16",
    // then every scale-folded dec.* tensor (name, data, count), then prepare.
    bool load(int device, const std::string &ftype, int max_batch, std::string &err) {
        release();
        const int dt = ftype == "f16" ? TPMD_DTYPE_F16 : TPMD_DTYPE_F32;
        if (ftype != "f16" && ftype != "f32") {
            err = "ftype must be f32 or f16";
            return false;
        }
        ctx = tpmd_create(device, dt, max_batch);
        if (!ctx) {
            err = tpmd_create_error();
            return false;
        }
        batch = max_batch;
        return true;
    }
    bool set_tensor(const std::string &name, const float *data, int64_t n, std::string &err) {
        return ok(tpmd_set_tensor(ctx, name.c_str(), data, n), err);
    }
    // the decoder's tensors straight from motion_ae_{f32,f16}.gguf (scale
    // folding included), in place of the set_tensor loop
    bool load_gguf(const std::string &path, std::string &err) {
        return ok(tpmd_load_gguf(ctx, path.c_str()), err);
    }
    bool prepare(std::string &err) { return ok(tpmd_prepare(ctx), err); }

    // motion_dec::build: the decode plan needs no graph construction here
    // (kernels are fixed; CUDA graphs are captured on first use)
    bool build(bool with_taps, std::string &err) {
        if (!ctx) {
            err = "decoder not loaded";
            return false;
        }
        (void) with_taps;
        built = true;
        taps_in_graph = false;
        return true;
    }
    // motion_dec::set_feats: feats[j] = [r*r][ST_OC[j]] channel-last f32
    bool set_feats(const std::vector<std::vector<float>> &feats, std::string &err) {
        if (feats.size() != TPMD_N_LEVELS) {
            err = "feat size mismatch";
            return false;
        }
        const float *p[TPMD_N_LEVELS];
        for (int j = 0; j < TPMD_N_LEVELS; j++) p[j] = feats[(size_t) j].data();
        return ok(tpmd_set_feats(ctx, p), err);
    }
    // motion_dec::decode_batch: styles [batch*512] -> imgs [batch*3*512*512]
    bool decode_batch(const float *styles, float *imgs_out, std::string &err) {
        return ok(tpmd_decode(ctx, styles, batch, imgs_out), err);
    }
    void release() {
        tpmd_destroy(ctx);
        ctx = nullptr;
        built = false;
    }

private:
    bool ok(int rc, std::string &err) {
        if (rc == 0) return true;
        err = tpmd_last_error(ctx);
        return false;
    }
};

}  // namespace tpmd_cpp
