// tpmd_group: the decoder on several GPUs behind the C ABI (include/tpmd.h).
//
// The reference decodes on one backend (src/pipeline.cpp:153-184,
// src/backend.cpp:9-57); frames are independent given the prepared weights
// and the portrait's feature pyramid, so the decoder shards by frame:
//
//  * a group owns one tpmd_ctx and one NCCL communicator per local GPU, in a
//    clique of `nranks` GPUs that one process (tpmd_group_create) or one
//    process per GPU (tpmd_group_create_rank) forms;
//  * global rank 0 holds the host weights and feats; prepare / set_feats run
//    there and the two device arenas go to every other rank by one
//    ncclBroadcast each (NVLink / NVSwitch), behind a broadcast status word
//    so a failure on rank 0 fails every rank instead of leaving it waiting;
//  * a decode of n frames gives rank r the contiguous frames
//    [r*ceil(n/P), (r+1)*ceil(n/P)) and writes them straight into the
//    caller's frame buffer; there is no collective on the data path;
//  * NCCL is loaded at run time (dlopen), communicators are created
//    non-blocking, and every wait on them (initialisation, a collective's
//    completion) is polled under a wall-clock limit (TPMD_NCCL_TIMEOUT_S,
//    default 120 s); on expiry or an asynchronous error the group aborts its
//    communicators and reports the failure.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <thread>
#include <vector>

#include "../../include/tpmd.h"

namespace {

thread_local std::string g_group_create_err;

// the NCCL entry points the group uses; the real table comes from dlopen,
// tests substitute a fake one (tpmd_group_selftest_nccl)
struct nccl_api {
    ncclResult_t (*get_unique_id)(ncclUniqueId *);
    ncclResult_t (*init_rank_config)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *);
    ncclResult_t (*get_async_error)(ncclComm_t, ncclResult_t *);
    ncclResult_t (*abort)(ncclComm_t);
    ncclResult_t (*destroy)(ncclComm_t);
    ncclResult_t (*group_start)();
    ncclResult_t (*group_end)();
    ncclResult_t (*broadcast)(const void *, void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t);
    const char *(*error_string)(ncclResult_t);
    int (*set_device)(int);  // cudaSetDevice; a fake table needs no GPU
};

std::mutex g_nccl_mu;
bool g_nccl_tried = false;
nccl_api g_nccl{};
std::string g_nccl_err;

int real_set_device(int d) { return (int) cudaSetDevice(d); }

// the process's NCCL (the one already loaded, e.g. by torch, else the
// system's libnccl.so.2)
const nccl_api *load_nccl(std::string &err) {
    std::lock_guard<std::mutex> lk(g_nccl_mu);
    if (!g_nccl_tried) {
        g_nccl_tried = true;
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            g_nccl_err = std::string("NCCL unavailable: ") + dlerror();
        } else {
            auto sym = [&](const char *n) {
                void *p = dlsym(h, n);
                if (!p && g_nccl_err.empty()) g_nccl_err = std::string("NCCL symbol missing: ") + n;
                return p;
            };
            g_nccl.get_unique_id = (decltype(g_nccl.get_unique_id)) sym("ncclGetUniqueId");
            g_nccl.init_rank_config = (decltype(g_nccl.init_rank_config)) sym("ncclCommInitRankConfig");
            g_nccl.get_async_error = (decltype(g_nccl.get_async_error)) sym("ncclCommGetAsyncError");
            g_nccl.abort = (decltype(g_nccl.abort)) sym("ncclCommAbort");
            g_nccl.destroy = (decltype(g_nccl.destroy)) sym("ncclCommDestroy");
            g_nccl.group_start = (decltype(g_nccl.group_start)) sym("ncclGroupStart");
            g_nccl.group_end = (decltype(g_nccl.group_end)) sym("ncclGroupEnd");
            g_nccl.broadcast = (decltype(g_nccl.broadcast)) sym("ncclBroadcast");
            g_nccl.all_reduce = (decltype(g_nccl.all_reduce)) sym("ncclAllReduce");
            g_nccl.error_string = (decltype(g_nccl.error_string)) sym("ncclGetErrorString");
            g_nccl.set_device = real_set_device;
        }
    }
    if (!g_nccl_err.empty()) {
        err = g_nccl_err;
        return nullptr;
    }
    return &g_nccl;
}

double timeout_s() {
    const char *e = getenv("TPMD_NCCL_TIMEOUT_S");
    const double v = e ? atof(e) : 120.0;
    return v > 0 ? v : 120.0;
}

using clk = std::chrono::steady_clock;
double since(clk::time_point t0) { return std::chrono::duration<double>(clk::now() - t0).count(); }

std::string nccl_msg(const nccl_api &api, const char *what, ncclResult_t r) {
    return std::string(what) + ": " + (api.error_string ? api.error_string(r) : "NCCL error") + " (" +
           std::to_string((int) r) + ")";
}

void abort_all(const nccl_api &api, std::vector<ncclComm_t> &comms, int *aborted) {
    for (ncclComm_t c : comms) {
        api.abort(c);
        if (aborted) ++*aborted;
    }
    comms.clear();
}

// Wait until no communicator has work in progress (ncclCommGetAsyncError),
// polling under the wall-clock limit; on expiry or an asynchronous error,
// abort them all. `aborted` counts the aborts issued.
bool settle(const nccl_api &api, std::vector<ncclComm_t> &comms, double limit, const char *what,
            std::string &err, int *aborted) {
    const clk::time_point t0 = clk::now();
    for (;;) {
        bool busy = false;
        for (ncclComm_t c : comms) {
            ncclResult_t st = ncclSuccess;
            const ncclResult_t r = api.get_async_error(c, &st);
            if (r != ncclSuccess) st = r;
            if (st == ncclInProgress) {
                busy = true;
            } else if (st != ncclSuccess) {
                err = nccl_msg(api, what, st);
                abort_all(api, comms, aborted);
                return false;
            }
        }
        if (!busy) return true;
        if (since(t0) > limit) {
            err = std::string(what) + ": timed out after " + std::to_string((int) limit) + " s";
            abort_all(api, comms, aborted);
            return false;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
}

// One non-blocking communicator per local device: local device i is global
// rank rank0 + i of nranks. Returns false (with every created communicator
// aborted) on an error or when initialisation does not finish in time.
bool init_comms(const nccl_api &api, const std::vector<int> &devs, int rank0, int nranks, const ncclUniqueId &id,
                double limit, std::vector<ncclComm_t> &comms, std::string &err, int *aborted) {
    comms.assign(devs.size(), nullptr);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = api.group_start();
    for (size_t i = 0; i < devs.size() && r == ncclSuccess; i++) {
        if (api.set_device(devs[i]) != 0) {
            err = "cudaSetDevice failed for device " + std::to_string(devs[i]);
            api.group_end();
            comms.clear();
            return false;
        }
        r = api.init_rank_config(&comms[i], nranks, id, rank0 + (int) i, &cfg);
        if (r == ncclInProgress) r = ncclSuccess;
    }
    const ncclResult_t e = api.group_end();
    if (r == ncclSuccess && e != ncclSuccess && e != ncclInProgress) r = e;
    std::vector<ncclComm_t> made;
    for (ncclComm_t c : comms)
        if (c) made.push_back(c);
    comms = made;
    if (r != ncclSuccess) {
        err = nccl_msg(api, "ncclCommInitRankConfig", r);
        abort_all(api, comms, aborted);
        return false;
    }
    return settle(api, comms, limit, "NCCL communicator initialisation", err, aborted);
}

}  // namespace

struct tpmd_group {
    std::vector<tpmd_ctx *> m;  // one decoder per local GPU
    std::vector<int> dev;
    std::vector<cudaStream_t> st;
    std::vector<void *> scratch;  // per member: 2 doubles (max) + a status int
    int rank0 = 0, nranks = 1;    // global rank of member 0, clique size
    const nccl_api *api = nullptr;
    std::vector<ncclComm_t> comms;
    bool prepared = false;
    std::string err;

    int root_local() const { return rank0 == 0 ? 0 : -1; }  // member that is global rank 0
    bool fail(const std::string &e) {
        err = e;
        return false;
    }
    bool ck(cudaError_t e, const char *what) {
        return e == cudaSuccess || fail(std::string(what) + ": " + cudaGetErrorString(e));
    }
    bool member_fail(int i, const char *what) {
        return fail(std::string(what) + " (device " + std::to_string(dev[(size_t) i]) +
                    "): " + tpmd_last_error(m[(size_t) i]));
    }

    // every member's stream drained, under the wall-clock limit (an abort of
    // the communicators ends collectives that can never complete)
    bool drain(const char *what) {
        const clk::time_point t0 = clk::now();
        const double limit = timeout_s();
        for (size_t i = 0; i < m.size(); i++) {
            if (!ck(cudaSetDevice(dev[i]), "cudaSetDevice")) return false;
            for (;;) {
                const cudaError_t q = cudaStreamQuery(st[i]);
                if (q == cudaSuccess) break;
                if (q != cudaErrorNotReady) return ck(q, what);
                if (since(t0) > limit) {
                    if (api) abort_all(*api, comms, nullptr);
                    return fail(std::string(what) + ": timed out after " + std::to_string((int) limit) + " s");
                }
                std::this_thread::sleep_for(std::chrono::microseconds(100));
            }
        }
        return true;
    }

    // bytes of member 0's buffer (global rank 0) to the same buffer on every rank
    bool bcast(const std::vector<void *> &bufs, size_t bytes, const char *what) {
        if (nranks == 1) return true;
        if (comms.size() != m.size()) return fail(std::string(what) + ": communicators were aborted");
        ncclResult_t r = api->group_start();
        for (size_t i = 0; i < m.size() && (r == ncclSuccess || r == ncclInProgress); i++)
            r = api->broadcast(bufs[i], bufs[i], bytes, ncclUint8, 0, comms[i], st[i]);
        const ncclResult_t e = api->group_end();
        if ((r != ncclSuccess && r != ncclInProgress) || (e != ncclSuccess && e != ncclInProgress))
            return fail(nccl_msg(*api, what, r != ncclSuccess && r != ncclInProgress ? r : e));
        std::string se;
        if (!settle(*api, comms, timeout_s(), what, se, nullptr)) return fail(se);
        return drain(what);
    }

    // status word of global rank 0 to every rank: true when rank 0 succeeded
    bool bcast_status(bool ok_here, const char *what) {
        if (nranks == 1) return ok_here;
        std::vector<void *> b(m.size());
        for (size_t i = 0; i < m.size(); i++) {
            b[i] = (char *) scratch[i] + 16;
            const int v = (root_local() == (int) i) ? (ok_here ? 1 : 0) : 0;
            if (!ck(cudaSetDevice(dev[i]), "cudaSetDevice") ||
                !ck(cudaMemcpyAsync(b[i], &v, 4, cudaMemcpyHostToDevice, st[i]), "status H2D"))
                return false;
        }
        // rank 0's own failure message is already in err; keep it
        const std::string own = err;
        if (!drain(what) || !bcast(b, 4, what)) return false;
        int v = 0;
        if (!ck(cudaSetDevice(dev[0]), "cudaSetDevice") ||
            !ck(cudaMemcpy(&v, b[0], 4, cudaMemcpyDeviceToHost), "status D2H"))
            return false;
        if (!ok_here) return fail(own);
        return v != 0 || fail(std::string(what) + ": failed on rank 0");
    }

    // arena `which` (0 weights, 1 feats) from global rank 0 to every rank
    bool share_arena(int which, bool ok_here, const char *what) {
        if (!bcast_status(ok_here, what)) return false;
        if (nranks == 1) return true;
        std::vector<void *> bufs(m.size());
        size_t bytes = 0;
        for (size_t i = 0; i < m.size(); i++)
            if (tpmd_arena(m[i], which, &bufs[i], &bytes) != 0) return member_fail((int) i, what);
        if (!bcast(bufs, bytes, what)) return false;
        for (size_t i = 0; i < m.size(); i++)
            if ((int) i != root_local() && tpmd_arena_adopt(m[i], which) != 0) return member_fail((int) i, what);
        return true;
    }

    ~tpmd_group() {
        if (api)
            for (ncclComm_t c : comms) api->destroy(c);
        for (size_t i = 0; i < m.size(); i++) {
            cudaSetDevice(dev[i]);
            if (st.size() > i && st[i]) cudaStreamDestroy(st[i]);
            if (scratch.size() > i && scratch[i]) cudaFree(scratch[i]);
            tpmd_destroy(m[i]);
        }
    }
};

namespace {

tpmd_group *make_group(const int *devices, int n, int rank0, int nranks, const void *id, int dtype,
                       int max_batch) {
    if (!devices || n < 1 || nranks < n || rank0 < 0 || rank0 + n > nranks) {
        g_group_create_err = "tpmd_group: bad device list or rank layout";
        return nullptr;
    }
    tpmd_group *g = new (std::nothrow) tpmd_group();
    if (!g) {
        g_group_create_err = "tpmd_group: out of host memory";
        return nullptr;
    }
    g->rank0 = rank0;
    g->nranks = nranks;
    for (int i = 0; i < n; i++) {
        tpmd_ctx *c = tpmd_create(devices[i], dtype, max_batch);
        if (!c) {
            g_group_create_err = std::string("tpmd_group: device ") + std::to_string(devices[i]) + ": " +
                                 tpmd_create_error();
            delete g;
            return nullptr;
        }
        g->m.push_back(c);
        g->dev.push_back(devices[i]);
        cudaStream_t s = nullptr;
        void *p = nullptr;
        if (cudaSetDevice(devices[i]) != cudaSuccess ||
            cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess ||
            cudaMalloc(&p, 256) != cudaSuccess) {
            g_group_create_err = "tpmd_group: stream or scratch on device " + std::to_string(devices[i]);
            if (s) cudaStreamDestroy(s);
            delete g;
            return nullptr;
        }
        g->st.push_back(s);
        g->scratch.push_back(p);
    }
    if (nranks > 1) {
        std::string e;
        g->api = load_nccl(e);
        ncclUniqueId uid;
        if (g->api && id)
            memcpy(&uid, id, sizeof uid);
        else if (g->api && g->api->get_unique_id(&uid) != ncclSuccess)
            e = "ncclGetUniqueId failed";
        if (!g->api || !e.empty() ||
            !init_comms(*g->api, g->dev, rank0, nranks, uid, timeout_s(), g->comms, e, nullptr)) {
            g_group_create_err = "tpmd_group: " + e;
            g->comms.clear();
            delete g;
            return nullptr;
        }
    }
    return g;
}

}  // namespace

extern "C" {

tpmd_group *tpmd_group_create(const int *devices, int n, int dtype, int max_batch) {
    return make_group(devices, n, 0, n, nullptr, dtype, max_batch);
}

int tpmd_group_unique_id(void *id, size_t len) {
    if (!id || len < sizeof(ncclUniqueId)) return -1;
    std::string e;
    const nccl_api *api = load_nccl(e);
    if (!api) {
        g_group_create_err = e;
        return -1;
    }
    ncclUniqueId u;
    if (api->get_unique_id(&u) != ncclSuccess) {
        g_group_create_err = "ncclGetUniqueId failed";
        return -1;
    }
    memcpy(id, &u, sizeof u);
    return 0;
}

tpmd_group *tpmd_group_create_rank(int device, int rank, int nranks, const void *id, size_t id_len, int dtype,
                                   int max_batch) {
    if (nranks > 1 && (!id || id_len < sizeof(ncclUniqueId))) {
        g_group_create_err = "tpmd_group_create_rank: missing NCCL unique id";
        return nullptr;
    }
    return make_group(&device, 1, rank, nranks, id, dtype, max_batch);
}

const char *tpmd_group_create_error(void) { return g_group_create_err.c_str(); }
void tpmd_group_destroy(tpmd_group *g) { delete g; }
const char *tpmd_group_last_error(const tpmd_group *g) { return g ? g->err.c_str() : "no group"; }
int tpmd_group_size(const tpmd_group *g) { return g ? (int) g->m.size() : -1; }
int tpmd_group_ranks(const tpmd_group *g, int *rank0, int *nranks) {
    if (!g) return -1;
    if (rank0) *rank0 = g->rank0;
    if (nranks) *nranks = g->nranks;
    return 0;
}
tpmd_ctx *tpmd_group_member(tpmd_group *g, int i) {
    return g && i >= 0 && i < (int) g->m.size() ? g->m[(size_t) i] : nullptr;
}

int tpmd_group_set_tensor(tpmd_group *g, const char *name, const float *data, int64_t n) {
    if (!g) return -1;
    const int r = g->root_local();
    if (r < 0) return 0;  // weights are read on global rank 0 only
    return tpmd_set_tensor(g->m[(size_t) r], name, data, n) == 0 ? 0 : (g->member_fail(r, "set_tensor"), -1);
}

int tpmd_group_load_gguf(tpmd_group *g, const char *path) {
    if (!g) return -1;
    const int r = g->root_local();
    if (r < 0) return 0;
    return tpmd_load_gguf(g->m[(size_t) r], path) == 0 ? 0 : (g->member_fail(r, "load_gguf"), -1);
}

int tpmd_group_prepare(tpmd_group *g) {
    if (!g) return -1;
    const int r = g->root_local();
    bool ok = true;
    if (r >= 0 && tpmd_prepare(g->m[(size_t) r]) != 0) ok = g->member_fail(r, "prepare");
    if (!g->share_arena(0, ok, "weights broadcast")) return -1;
    g->prepared = true;
    return 0;
}

int tpmd_group_set_feats(tpmd_group *g, const float *const feats[TPMD_N_LEVELS]) {
    if (!g) return -1;
    const int r = g->root_local();
    bool ok = true;
    if (r >= 0 && tpmd_set_feats(g->m[(size_t) r], feats) != 0) ok = g->member_fail(r, "set_feats");
    return g->share_arena(1, ok, "feats broadcast") ? 0 : -1;
}

int tpmd_group_set_feats_device(tpmd_group *g, const float *const feats_dev[TPMD_N_LEVELS], void *stream) {
    if (!g) return -1;
    const int r = g->root_local();
    bool ok = true;
    if (r >= 0 && tpmd_set_feats_device(g->m[(size_t) r], feats_dev, stream) != 0)
        ok = g->member_fail(r, "set_feats_device");
    return g->share_arena(1, ok, "feats broadcast") ? 0 : -1;
}

int tpmd_shard_range(int64_t n, int nranks, int rank, int64_t *lo, int64_t *hi) {
    if (n < 0 || nranks < 1 || rank < 0 || rank >= nranks || !lo || !hi) return -1;
    const int64_t per = (n + nranks - 1) / nranks;
    *lo = std::min<int64_t>(n, (int64_t) rank * per);
    *hi = std::min<int64_t>(n, *lo + per);
    return 0;
}

}  // extern "C"

namespace {
// each local GPU decodes its shard on its own host thread into its slice of
// the caller's buffer (f32 CHW frames, or RGB24 bytes)
int group_decode(tpmd_group *g, const float *styles, int64_t n, void *out, bool rgb, const char *who) {
    if (!g) return -1;
    if (!styles || !out || n < 1) return g->fail(std::string(who) + ": bad argument"), -1;
    const size_t fsz = (size_t) 3 * TPMD_IMG * TPMD_IMG * (rgb ? 1 : 4);  // bytes per frame
    std::vector<int> rc(g->m.size(), 0);
    std::vector<std::thread> th;
    for (size_t i = 0; i < g->m.size(); i++) {
        int64_t lo = 0, hi = 0;
        tpmd_shard_range(n, g->nranks, g->rank0 + (int) i, &lo, &hi);
        if (hi <= lo) continue;
        th.emplace_back([&, i, lo, hi] {
            const float *s = styles + (size_t) lo * TPMD_STYLE_DIM;
            char *o = (char *) out + (size_t) lo * fsz;
            rc[i] = rgb ? tpmd_decode_rgb24(g->m[i], s, hi - lo, (uint8_t *) o)
                        : tpmd_decode(g->m[i], s, hi - lo, (float *) o);
        });
    }
    for (auto &t : th) t.join();
    for (size_t i = 0; i < g->m.size(); i++)
        if (rc[i] != 0) return g->member_fail((int) i, who), -1;
    return 0;
}
}  // namespace

extern "C" {

int tpmd_group_decode(tpmd_group *g, const float *styles, int64_t n, float *frames) {
    return group_decode(g, styles, n, frames, false, "tpmd_group_decode");
}

int tpmd_group_decode_rgb24(tpmd_group *g, const float *styles, int64_t n, uint8_t *rgb) {
    return group_decode(g, styles, n, rgb, true, "tpmd_group_decode_rgb24");
}

int tpmd_group_max(tpmd_group *g, double value, double *out) {
    if (!g || !out) return -1;
    if (g->nranks == 1 && g->m.size() == 1) {
        *out = value;
        return 0;
    }
    std::vector<void *> b(g->m.size());
    for (size_t i = 0; i < g->m.size(); i++) {
        b[i] = g->scratch[i];
        if (!g->ck(cudaSetDevice(g->dev[i]), "cudaSetDevice") ||
            !g->ck(cudaMemcpyAsync(b[i], &value, 8, cudaMemcpyHostToDevice, g->st[i]), "max H2D"))
            return -1;
    }
    if (!g->drain("max over ranks")) return -1;
    if (g->nranks > 1) {
        if (g->comms.size() != g->m.size()) return g->fail("max over ranks: communicators were aborted"), -1;
        ncclResult_t r = g->api->group_start();
        for (size_t i = 0; i < g->m.size() && (r == ncclSuccess || r == ncclInProgress); i++)
            r = g->api->all_reduce(b[i], b[i], 1, ncclFloat64, ncclMax, g->comms[i], g->st[i]);
        const ncclResult_t e = g->api->group_end();
        if ((r != ncclSuccess && r != ncclInProgress) || (e != ncclSuccess && e != ncclInProgress))
            return g->fail(nccl_msg(*g->api, "max over ranks", r)), -1;
        std::string se;
        if (!settle(*g->api, g->comms, timeout_s(), "max over ranks", se, nullptr)) return g->fail(se), -1;
        if (!g->drain("max over ranks")) return -1;
    }
    double v = value;
    if (!g->ck(cudaSetDevice(g->dev[0]), "cudaSetDevice") ||
        !g->ck(cudaMemcpy(&v, b[0], 8, cudaMemcpyDeviceToHost), "max D2H"))
        return -1;
    *out = v;
    return 0;
}

// Runs the communicator set-up and its failure handling against a fake NCCL
// (no GPU): scenario 0 initialises after a few polls, 1 never finishes (the
// wall-clock limit expires), 2 reports an asynchronous error on the last
// rank, 3 fails the init call itself. Returns 0 or -1 with the message in
// err; *aborted counts the ncclCommAbort calls.
int tpmd_group_selftest_nccl(int n, int scenario, double limit_s, int *aborted, char *err, size_t err_len) {
    struct fake {
        static int &scen() {
            static thread_local int s = 0;
            return s;
        }
        static int &polls() {
            static thread_local int p = 0;
            return p;
        }
        static ncclResult_t uid(ncclUniqueId *u) {
            memset(u, 0, sizeof *u);
            return ncclSuccess;
        }
        static ncclResult_t init(ncclComm_t *c, int, ncclUniqueId, int rank, ncclConfig_t *cfg) {
            if (scen() == 3 && rank == 1) return ncclInvalidArgument;
            if (!cfg || cfg->blocking != 0) return ncclInvalidArgument;  // must be non-blocking
            *c = (ncclComm_t) (intptr_t) (rank + 1);
            return ncclInProgress;
        }
        static ncclResult_t async(ncclComm_t c, ncclResult_t *st) {
            const int rank = (int) (intptr_t) c - 1;
            const int p = ++polls();
            if (scen() == 1) *st = ncclInProgress;
            else if (scen() == 2 && rank > 0 && p > 4) *st = ncclSystemError;
            else *st = p > 6 ? ncclSuccess : ncclInProgress;
            return ncclSuccess;
        }
        static ncclResult_t ok0() { return ncclSuccess; }
        static ncclResult_t okc(ncclComm_t) { return ncclSuccess; }
        static const char *es(ncclResult_t) { return "fake NCCL error"; }
        static int setdev(int) { return 0; }
    };
    fake::scen() = scenario;
    fake::polls() = 0;
    nccl_api api{};
    api.get_unique_id = fake::uid;
    api.init_rank_config = fake::init;
    api.get_async_error = fake::async;
    api.abort = fake::okc;
    api.destroy = fake::okc;
    api.group_start = fake::ok0;
    api.group_end = fake::ok0;
    api.error_string = fake::es;
    api.set_device = fake::setdev;
    std::vector<int> devs((size_t) std::max(1, n));
    for (size_t i = 0; i < devs.size(); i++) devs[i] = (int) i;
    ncclUniqueId id;
    fake::uid(&id);
    std::vector<ncclComm_t> comms;
    std::string e;
    int ab = 0;
    const bool ok = init_comms(api, devs, 0, (int) devs.size(), id, limit_s, comms, e, &ab);
    if (aborted) *aborted = ab;
    if (err && err_len) snprintf(err, err_len, "%s", e.c_str());
    return ok ? 0 : -1;
}

}  // extern "C"
