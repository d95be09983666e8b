// GGUF v3 reader for the motion_ae weight file: the on-disk step in front of
// the decoder (src/gguf_load.cpp:50-197, called from src/tp.cpp:32-36 with
// architecture "float-motion-ae" and motion_ae_scale).
//
// File layout (GGUF v3, little endian): "GGUF", u32 version, u64 tensor
// count, u64 key/value count; the key/value pairs (u64-length strings, u32
// value type, value); per tensor: name, u32 dims, u64 dim sizes (ggml order,
// fastest first), u32 element type, u64 offset into the data section; the
// data section starts at the next multiple of 32 bytes after the tensor
// infos.
//
// Accepted exactly as the reference accepts them: version 3; at most 100000
// tensors and 100000 keys; value types u32 (4), i32 (5), f32 (6), bool (7)
// and string (8); element types f32 (0) and f16 (1); up to 8 dims of which
// at most 4 are not 1 (unit dims are kept in order while fewer than 4 dims
// are recorded, later ones dropped: the 5-D modconv weights [k,k,IC,OC,1]
// become [k,k,IC,OC]). Every tensor is delivered as f32, times the
// motion_ae_scale factor of (name, dims) when folding is on, exactly as the
// reference's host copies are formed (f16 -> f32 exactly, then a float
// multiply by (float) scale).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include <cuda_fp16.h>

#include "../../include/tpmd.h"

namespace {

struct mapped_file {
    const uint8_t *p = nullptr;
    size_t n = 0;
    bool open(const char *path, std::string &err) {
        const int fd = ::open(path, O_RDONLY);
        if (fd < 0) {
            err = std::string(path) + ": cannot open";
            return false;
        }
        struct stat st{};
        if (fstat(fd, &st) != 0) {
            ::close(fd);
            err = std::string(path) + ": cannot stat";
            return false;
        }
        n = (size_t) st.st_size;
        if (n > 0) {
            void *m = mmap(nullptr, n, PROT_READ, MAP_PRIVATE, fd, 0);
            if (m == MAP_FAILED) {
                ::close(fd);
                err = std::string(path) + ": cannot map";
                return false;
            }
            p = (const uint8_t *) m;
        }
        ::close(fd);
        return true;
    }
    ~mapped_file() {
        if (p) munmap((void *) p, n);
    }
};

// bounds-checked little-endian cursor; `ok` turns false on the first overrun
struct cursor {
    const uint8_t *p, *end;
    bool ok = true;
    template <typename T>
    T get() {
        T v{};
        if ((size_t) (end - p) < sizeof(T)) {
            ok = false;
            return v;
        }
        memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t len = get<uint64_t>();
        if (!ok || len > (uint64_t) (end - p) || len > (1u << 20)) {
            ok = false;
            return {};
        }
        std::string s((const char *) p, (size_t) len);
        p += len;
        return s;
    }
};

struct tensor_info {
    std::string name;
    int64_t ne[4] = {1, 1, 1, 1};
    uint32_t type = 0;
    uint64_t offset = 0;
    int64_t count = 1;
};

void put_err(char *buf, size_t len, const std::string &msg) {
    if (!buf || len == 0) return;
    const size_t k = msg.size() < len - 1 ? msg.size() : len - 1;
    memcpy(buf, msg.data(), k);
    buf[k] = 0;
}

int read_gguf(const char *path, const char *expect_arch, int fold, tpmd_gguf_tensor_fn cb, void *user,
              std::string &err, tpmd_gguf_kv_fn kv_cb = nullptr) {
    if (!path || (!cb && !kv_cb)) {
        err = "tpmd_gguf_read: null argument";
        return -1;
    }
    mapped_file f;
    if (!f.open(path, err)) return -1;
    const std::string P = path;
    cursor c{f.p, f.p + f.n};
    const uint32_t magic = c.get<uint32_t>();  // "GGUF" as little-endian bytes
    if (!c.ok || memcmp(&magic, "GGUF", 4) != 0) {
        err = P + ": not a GGUF file";
        return -1;
    }
    if (c.get<uint32_t>() != 3) {
        err = P + ": unsupported GGUF version";
        return -1;
    }
    const uint64_t n_tensors = c.get<uint64_t>();
    const uint64_t n_kv = c.get<uint64_t>();
    if (!c.ok || n_tensors > 100000 || n_kv > 100000) {
        err = P + ": corrupt header";
        return -1;
    }
    std::string arch;
    bool have_arch = false;
    for (uint64_t i = 0; i < n_kv && c.ok; i++) {
        const std::string key = c.str();
        const uint32_t vt = c.get<uint32_t>();
        double num = 0.0;
        std::string sv;
        switch (vt) {
            case 4: num = c.get<uint32_t>(); break;
            case 5: num = c.get<int32_t>(); break;
            case 6: num = c.get<float>(); break;
            case 7: num = c.get<uint8_t>() ? 1 : 0; break;
            case 8: {
                sv = c.str();
                if (key == "general.architecture") {
                    arch = sv;
                    have_arch = true;
                }
                break;
            }
            default:
                err = P + ": unsupported KV type " + std::to_string(vt) + " for " + key;
                return -1;
        }
        if (kv_cb && c.ok && kv_cb(user, key.c_str(), vt, num, vt == 8 ? sv.c_str() : nullptr) != 0) {
            err = P + ": key " + key + " rejected by the consumer";
            return -1;
        }
    }
    if (!c.ok) {
        err = P + ": truncated KV section";
        return -1;
    }
    if (expect_arch && (!have_arch || arch != expect_arch)) {
        err = P + ": unexpected architecture '" + (have_arch ? arch : std::string("<none>")) +
              "', want " + expect_arch;
        return -1;
    }
    if (!cb) return 0;  // key/value pairs only
    std::vector<tensor_info> infos((size_t) n_tensors);
    for (tensor_info &t : infos) {
        t.name = c.str();
        const uint32_t nd = c.get<uint32_t>();
        if (!c.ok || nd > 8) {
            err = P + ": corrupt tensor info";
            return -1;
        }
        int used = 0;
        for (uint32_t d = 0; d < nd; d++) {
            const uint64_t len = c.get<uint64_t>();
            if (len != 1) {
                if (used >= 4) {
                    err = P + ": tensor " + t.name + " has >4 non-unit dims";
                    return -1;
                }
                t.ne[used++] = (int64_t) len;
            } else if (used < 4) {
                t.ne[used++] = 1;
            }
            t.count *= (int64_t) (len ? len : 1);
            if (len > (1ull << 40) || t.count > (int64_t) 1 << 40) {  // no file holds that much
                err = P + ": corrupt tensor info";
                return -1;
            }
        }
        t.type = c.get<uint32_t>();
        t.offset = c.get<uint64_t>();
        if (t.type > 1) {
            err = P + ": tensor " + t.name + " has unsupported type";
            return -1;
        }
    }
    if (!c.ok) {
        err = P + ": truncated tensor info section";
        return -1;
    }
    const size_t data_off = ((size_t) (c.p - f.p) + 31) & ~(size_t) 31;
    std::vector<float> buf;
    for (const tensor_info &t : infos) {
        const size_t esz = t.type == 0 ? 4 : 2;
        const size_t bytes = (size_t) t.count * esz;
        if (t.offset > f.n || data_off > f.n - t.offset || bytes > f.n - data_off - t.offset) {
            err = P + ": tensor " + t.name + " out of bounds";
            return -1;
        }
        const uint8_t *src = f.p + data_off + t.offset;
        buf.resize((size_t) t.count);
        if (t.type == 0) {
            memcpy(buf.data(), src, bytes);
        } else {
            for (int64_t i = 0; i < t.count; i++) {
                __half_raw h;
                memcpy(&h.x, src + 2 * i, 2);
                buf[(size_t) i] = __half2float(__half(h));
            }
        }
        if (fold) {
            const double s = tpmd_scale_for(t.name.c_str(), t.ne);
            if (s != 1.0) {
                const float fs = (float) s;
                for (float &v : buf) v *= fs;
            }
        }
        const int rc = cb(user, t.name.c_str(), t.ne, buf.data(), t.count);
        if (rc != 0) {
            err = P + ": tensor " + t.name + " rejected by the consumer";
            return -1;
        }
    }
    return 0;
}

struct load_state {
    tpmd_ctx *ctx;
    int set = 0;
};

// decoder tensors only: "dec.*" without the motion direction basis (the
// encoder's half and dec.direction belong to the encoder and the pipeline)
int to_decoder(void *user, const char *name, const int64_t *, const float *data, int64_t n) {
    load_state *s = (load_state *) user;
    if (strncmp(name, "dec.", 4) != 0 || strncmp(name, "dec.direction", 13) == 0) return 0;
    if (tpmd_set_tensor(s->ctx, name, data, n) != 0) return -1;
    s->set++;
    return 0;
}

}  // namespace

// error text of a failed tpmd_load_gguf lives in the ctx (tpmd_api.cu)
__attribute__((visibility("hidden"))) int tpmd_ctx_fail(tpmd_ctx *ctx, const char *msg);

extern "C" {

int tpmd_gguf_read(const char *path, const char *expect_arch, int fold_scales, tpmd_gguf_tensor_fn cb,
                   void *user, char *err, size_t err_len) {
    std::string e;
    const int rc = read_gguf(path, expect_arch, fold_scales, cb, user, e);
    if (rc != 0) put_err(err, err_len, e);
    return rc;
}

int tpmd_gguf_read_kv(const char *path, const char *expect_arch, tpmd_gguf_kv_fn cb, void *user, char *err,
                      size_t err_len) {
    std::string e;
    if (!cb) {
        put_err(err, err_len, "tpmd_gguf_read_kv: null argument");
        return -1;
    }
    const int rc = read_gguf(path, expect_arch, 0, nullptr, user, e, cb);
    if (rc != 0) put_err(err, err_len, e);
    return rc;
}

int tpmd_load_gguf(tpmd_ctx *ctx, const char *path) {
    if (!ctx) return -1;
    load_state s{ctx};
    std::string e;
    if (read_gguf(path, "float-motion-ae", 1, to_decoder, &s, e) != 0) {
        // a tensor the decoder refused keeps tpmd_set_tensor's own message
        if (e.find("rejected by the consumer") == std::string::npos) tpmd_ctx_fail(ctx, e.c_str());
        return -1;
    }
    return 0;
}

}  // extern "C"
