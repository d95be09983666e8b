// C++ shim over tpmd.h with the method shape the reference's pipeline uses
// for its decoder (tp::motion_dec, src/motion_dec.h:10-49; called from
// src/pipeline.cpp:153-175): build / set_feats / decode_batch / batch /
// built / taps_in_graph, errors as bool + std::string. The call sites of
// pipeline.cpp compile unchanged: build, set_feats and decode_batch also
// accept the reference's argument lists (a backend argument, which the B200
// decoder does not need and ignores, and a menc_result-like object whose
// `feats` member holds the pyramid). One decoder may span several GPUs
// (load_devices): frames of a batch shard across them. Header-only; link
// libtpmd.so.
#pragma once

#include <cstring>
#include <string>
#include <utility>
#include <vector>

#include "tpmd.h"

namespace tpmd_cpp {

struct motion_dec_b200 {
    tpmd_group *group = nullptr;
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
        return load_devices(std::vector<int>{device}, ftype, max_batch, err);
    }
    // the same decoder on several GPUs of this process: a decode_batch call
    // splits its frames into contiguous shards, one per GPU
    bool load_devices(const std::vector<int> &devices, const std::string &ftype, int max_batch,
                      std::string &err) {
        release();
        if (ftype != "f16" && ftype != "f32") {
            err = "ftype must be f32 or f16";
            return false;
        }
        const int dt = ftype == "f16" ? TPMD_DTYPE_F16 : TPMD_DTYPE_F32;
        group = tpmd_group_create(devices.data(), (int) devices.size(), dt, max_batch);
        if (!group) {
            err = tpmd_group_create_error();
            return false;
        }
        batch = max_batch;
        return true;
    }
    bool set_tensor(const std::string &name, const float *data, int64_t n, std::string &err) {
        return ok(tpmd_group_set_tensor(group, name.c_str(), data, n), err);
    }
    // the decoder's tensors straight from motion_ae_{f32,f16}.gguf (scale
    // folding included), in place of the set_tensor loop
    bool load_gguf(const std::string &path, std::string &err) {
        return ok(tpmd_group_load_gguf(group, path.c_str()), err);
    }
    bool prepare(std::string &err) { return ok(tpmd_group_prepare(group), err); }

    // motion_dec::build: the decode plan needs no graph construction here
    // (kernels are fixed; CUDA graphs are captured on first use)
    bool build(bool with_taps, std::string &err) {
        if (!group) {
            err = "decoder not loaded";
            return false;
        }
        (void) with_taps;
        built = true;
        taps_in_graph = false;
        return true;
    }
    // the reference's signature, build(backend_t &, bool, std::string &)
    template <typename Backend>
    bool build(Backend &, bool with_taps, std::string &err) {
        return build(with_taps, err);
    }
    // motion_dec::set_feats: feats[j] = [r*r][ST_OC[j]] channel-last f32
    bool set_feats(const std::vector<std::vector<float>> &feats, std::string &err) {
        if (feats.size() != TPMD_N_LEVELS) {
            err = "feat size mismatch";
            return false;
        }
        const float *p[TPMD_N_LEVELS];
        for (int j = 0; j < TPMD_N_LEVELS; j++) p[j] = feats[(size_t) j].data();
        return ok(tpmd_group_set_feats(group, p), err);
    }
    // the reference's signature, set_feats(const menc_result &, std::string &)
    template <typename MencResult, typename = decltype(std::declval<const MencResult &>().feats)>
    bool set_feats(const MencResult &m, std::string &err) {
        return set_feats(m.feats, err);
    }
    // motion_dec::decode_batch: styles [batch*512] -> imgs [batch*3*512*512]
    bool decode_batch(const float *styles, float *imgs_out, std::string &err) {
        return ok(tpmd_group_decode(group, styles, batch, imgs_out), err);
    }
    // the reference's signature, decode_batch(backend_t &, styles, imgs, err)
    template <typename Backend>
    bool decode_batch(Backend &, const float *styles, float *imgs_out, std::string &err) {
        return decode_batch(styles, imgs_out, err);
    }
    // the decoder of GPU i (taps, device-pointer decodes, profiling)
    tpmd_ctx *member(int i = 0) const { return tpmd_group_member(group, i); }
    void release() {
        tpmd_group_destroy(group);
        group = nullptr;
        built = false;
    }

private:
    bool ok(int rc, std::string &err) {
        if (rc == 0) return true;
        err = group ? tpmd_group_last_error(group) : "decoder not loaded";
        return false;
    }
};

}  // namespace tpmd_cpp
