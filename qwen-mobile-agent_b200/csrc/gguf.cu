// gguf.cu -- the engine's GGUF v3 file reader: the header, the metadata the
// engine depends on, the tensor infos and the aligned data section, and a
// model load straight from a file.  This is the parsing half of qma_load
// (gguf.c:104-316); the tokenizer tables qma_load also builds stay with
// qma's host code (the engine consumes token ids).
//
// Differences from qma_load, on purpose: Q8_0 tensors are accepted (the
// engine computes with them; qma_load rejects type 8, gguf.c:275-281);
// the vocabulary size is taken from token_embd.weight, not capped by the
// reference's compile-time N_VOCAB; every read is bounds-checked, including
// the fixed-size values qma_load skips without a check.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"

namespace {

// GGUF metadata value types (the GGUF v3 format)
enum : uint32_t {
    GV_U8 = 0, GV_I8, GV_U16, GV_I16, GV_U32, GV_I32, GV_F32, GV_BOOL, GV_STR, GV_ARR, GV_U64, GV_I64, GV_F64
};

class Cursor {
  public:
    Cursor(const uint8_t *b, const uint8_t *e) : p_(b), e_(e) {}
    bool ok() const { return ok_; }
    const uint8_t *pos() const { return p_; }
    bool take(uint64_t n) {
        if (!ok_ || uint64_t(e_ - p_) < n) {
            ok_ = false;
            return false;
        }
        p_ += n;
        return true;
    }
    template <class T> T get() {
        T v{};
        if (take(sizeof(T))) memcpy(&v, p_ - sizeof(T), sizeof(T));
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!take(n)) return {};
        return std::string(reinterpret_cast<const char *>(p_ - n), size_t(n));
    }
    // an unsigned count: the unsigned widths and int32, as GGUF writers emit
    bool count(uint32_t t, uint64_t &out) {
        switch (t) {
        case GV_U8: out = get<uint8_t>(); return ok_;
        case GV_U16: out = get<uint16_t>(); return ok_;
        case GV_U32: out = get<uint32_t>(); return ok_;
        case GV_U64: out = get<uint64_t>(); return ok_;
        case GV_I32: out = uint64_t(int64_t(get<int32_t>())); return ok_;
        default: return false;
        }
    }
    void skip(uint32_t t, int depth = 0) {
        static const uint8_t width[] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
        if (t == GV_STR) {
            str();
        } else if (t == GV_ARR && depth < 4) {
            const uint32_t at = get<uint32_t>();
            const uint64_t n = get<uint64_t>();
            if (at != GV_STR && at != GV_ARR && at <= GV_F64) {
                if (n > uint64_t(e_ - p_) / width[at]) ok_ = false;
                else take(n * width[at]);
            } else {
                for (uint64_t i = 0; i < n && ok_; i++) skip(at, depth + 1);
            }
        } else if (t <= GV_F64 && width[t]) {
            take(width[t]);
        } else {
            ok_ = false;
        }
    }

  private:
    const uint8_t *p_, *e_;
    bool ok_ = true;
};

// The hyper-parameters the engine is built for (qma.h:28-37): 40 layers,
// embedding 2048, 16 / 2 heads, 64 rotary dims in sections 11 / 11 / 10.
struct Hparams {
    uint64_t block_count = 0, embd = 0, head = 0, head_kv = 0, n_rot = 0, sect[3] = {0, 0, 0};
    uint64_t alignment = 32, n_tokens = 0;
    bool matches() const {
        return block_count == 40 && embd == 2048 && head == 16 && head_kv == 2 && n_rot == 64 && sect[0] == 11 &&
               sect[1] == 11 && sect[2] == 10;
    }
};

// bytes of a tensor of type `type` with ne0 elements per row (0: unsupported
// type or a row that is not whole blocks)
uint64_t row_bytes(uint32_t type, int64_t ne0) {
    uint64_t bs, blk;
    switch (type) {
    case QMA_TYPE_F32: bs = 4; blk = 1; break;
    case QMA_TYPE_Q8_0: bs = 34; blk = 32; break;
    case QMA_TYPE_Q4_K: bs = 144; blk = 256; break;
    case QMA_TYPE_Q6_K: bs = 210; blk = 256; break;
    default: return 0;
    }
    if (ne0 <= 0 || uint64_t(ne0) % blk) return 0;
    return uint64_t(ne0) / blk * bs;
}

// Parses [base, base + size): tensors, the data section's offset in the
// file, the hyper-parameters.  Returns a status; the message says why.
int parse(const uint8_t *base, size_t size, std::vector<qma_cuda_tensor> &tensors, uint64_t &data_off,
          Hparams &hp) {
    if (size < 24 || memcmp(base, "GGUF", 4) != 0) {
        qma::set_error("gguf: not a GGUF file");
        return QMA_CUDA_ERR_INVALID;
    }
    Cursor c(base + 4, base + size);
    const uint32_t version = c.get<uint32_t>();
    const uint64_t n_tensors = c.get<uint64_t>(), n_kv = c.get<uint64_t>();
    if (version < 2) {
        qma::set_error("gguf: version %u (2 or 3 needed)", version);
        return QMA_CUDA_ERR_UNSUPPORTED;
    }
    for (uint64_t i = 0; i < n_kv && c.ok(); i++) {
        std::string key = c.str();
        const uint32_t t = c.get<uint32_t>();
        if (!c.ok()) break;
        // the architecture prefix is dropped (gguf.c:146-152)
        for (const char *arch : {"qwen35moe.", "qwen35."})
            if (key.compare(0, strlen(arch), arch) == 0) {
                key.erase(0, strlen(arch));
                break;
            }
        uint64_t *dst = key == "block_count" ? &hp.block_count
                        : key == "embedding_length" ? &hp.embd
                        : key == "attention.head_count" ? &hp.head
                        : key == "attention.head_count_kv" ? &hp.head_kv
                        : key == "rope.dimension_count" ? &hp.n_rot
                        : key == "general.alignment" ? &hp.alignment
                                                      : nullptr;
        if (dst) {
            uint64_t v;
            if (c.count(t, v)) *dst = v;
            else c.skip(t);
        } else if (key == "rope.dimension_sections" && t == GV_ARR) {
            const uint32_t at = c.get<uint32_t>();
            const uint64_t n = c.get<uint64_t>();
            for (uint64_t j = 0; j < n && c.ok(); j++) {
                uint64_t v = 0;
                if (!c.count(at, v)) {
                    c.skip(at);
                    v = 0;
                }
                if (j < 3) hp.sect[j] = v;
            }
        } else if (key == "tokenizer.ggml.tokens" && t == GV_ARR) {
            const uint32_t at = c.get<uint32_t>();
            const uint64_t n = c.get<uint64_t>();
            hp.n_tokens = n;
            for (uint64_t j = 0; j < n && c.ok(); j++) c.skip(at);
        } else {
            c.skip(t);
        }
    }
    if (!c.ok()) {
        qma::set_error("gguf: corrupt metadata");
        return QMA_CUDA_ERR_INVALID;
    }
    if (!hp.matches()) {
        qma::set_error("gguf: hyper-parameters mismatch: the engine runs qwen35moe with 40 layers, embedding 2048, "
                       "heads 16/2, 64 rotary dims in sections 11/11/10; the file has %llu layers, embedding %llu, "
                       "heads %llu/%llu, %llu rotary dims in sections %llu/%llu/%llu",
                       (unsigned long long)hp.block_count, (unsigned long long)hp.embd,
                       (unsigned long long)hp.head, (unsigned long long)hp.head_kv, (unsigned long long)hp.n_rot,
                       (unsigned long long)hp.sect[0], (unsigned long long)hp.sect[1],
                       (unsigned long long)hp.sect[2]);
        return QMA_CUDA_ERR_UNSUPPORTED;
    }
    if (hp.alignment == 0 || hp.alignment > (1u << 20)) {
        qma::set_error("gguf: alignment %llu", (unsigned long long)hp.alignment);
        return QMA_CUDA_ERR_INVALID;
    }
    if (n_tensors > size / 24) {
        qma::set_error("gguf: corrupt tensor info (%llu tensors)", (unsigned long long)n_tensors);
        return QMA_CUDA_ERR_INVALID;
    }
    tensors.assign(size_t(n_tensors), qma_cuda_tensor{});
    for (auto &t : tensors) {
        const std::string name = c.str();
        snprintf(t.name, sizeof t.name, "%s", name.c_str());
        const uint32_t nd = c.get<uint32_t>();
        if (nd > 8) c.take(~uint64_t(0));              // corrupt: stop
        t.ne[0] = t.ne[1] = t.ne[2] = 1;
        for (uint32_t d = 0; d < nd && c.ok(); d++) {
            const uint64_t v = c.get<uint64_t>();
            if (d < 3) t.ne[d] = int64_t(v);            // further dims ignored (gguf.c:290)
        }
        t.type = c.get<uint32_t>();
        t.off = c.get<uint64_t>();
        if (!c.ok()) break;
    }
    if (!c.ok()) {
        qma::set_error("gguf: corrupt tensor info");
        return QMA_CUDA_ERR_INVALID;
    }
    const uint64_t here = uint64_t(c.pos() - base);
    data_off = (here + hp.alignment - 1) / hp.alignment * hp.alignment;
    const uint64_t avail = size > data_off ? size - data_off : 0;
    for (auto &t : tensors) {
        const uint64_t rb = row_bytes(t.type, t.ne[0]);
        if (!rb) {
            qma::set_error("gguf: tensor %s: type %u with rows of %lld elements is not supported", t.name, t.type,
                           (long long)t.ne[0]);
            return QMA_CUDA_ERR_UNSUPPORTED;
        }
        if (t.ne[0] < 1 || t.ne[1] < 1 || t.ne[2] < 1 || t.ne[0] > INT32_MAX || t.ne[1] > INT32_MAX ||
            t.ne[2] > INT32_MAX) {
            qma::set_error("gguf: tensor %s: bad shape", t.name);
            return QMA_CUDA_ERR_INVALID;
        }
        // the product rb * ne1 * ne2 is formed only once each factor is known
        // to fit in the file, so it cannot wrap around
        const uint64_t ne1 = uint64_t(t.ne[1]), ne2 = uint64_t(t.ne[2]);
        if (t.off > avail || ne1 > (avail - t.off) / rb || ne2 > (avail - t.off) / (rb * ne1)) {
            qma::set_error("gguf: tensor %s lies outside the file", t.name);
            return QMA_CUDA_ERR_INVALID;
        }
        t.nbytes = rb * ne1 * ne2;
        if (t.nbytes > avail - t.off) {
            qma::set_error("gguf: tensor %s lies outside the file", t.name);
            return QMA_CUDA_ERR_INVALID;
        }
    }
    return QMA_CUDA_OK;
}

// A read-only mapping of a whole file.
struct Mapping {
    int fd = -1;
    void *p = MAP_FAILED;
    size_t size = 0;
    int open(const char *path) {
        fd = ::open(path, O_RDONLY);
        struct stat st;
        if (fd < 0 || fstat(fd, &st) != 0) {
            qma::set_error("gguf: cannot open %s", path);
            return QMA_CUDA_ERR_INVALID;
        }
        size = size_t(st.st_size);
        if (size) p = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
        if (p == MAP_FAILED) {
            qma::set_error("gguf: cannot map %s (%zu bytes)", path, size);
            return QMA_CUDA_ERR_NOMEM;
        }
        return QMA_CUDA_OK;
    }
    ~Mapping() {
        if (p != MAP_FAILED) munmap(p, size);
        if (fd >= 0) close(fd);
    }
};

}  // namespace

extern "C" {

int qma_cuda_gguf_scan(const char *path, qma_cuda_tensor *tensors, uint32_t cap, uint32_t *n_tensors,
                       uint64_t *data_offset, uint64_t *n_tokens) {
    qma::clear_error();
    QMA_REQUIRE(path && n_tensors && (tensors || cap == 0), "qma_cuda_gguf_scan: bad arguments");
    Mapping f;
    int rc = f.open(path);
    if (rc) return rc;
    std::vector<qma_cuda_tensor> t;
    uint64_t off = 0;
    Hparams hp;
    if ((rc = parse(static_cast<const uint8_t *>(f.p), f.size, t, off, hp))) return rc;
    *n_tensors = uint32_t(t.size());
    for (uint32_t i = 0; i < cap && i < t.size(); i++) tensors[i] = t[i];
    if (data_offset) *data_offset = off;
    if (n_tokens) *n_tokens = hp.n_tokens;
    return QMA_CUDA_OK;
}

int qma_cuda_model_load_gguf(int device, const char *path, qma_cuda_model **out) {
    qma::clear_error();
    QMA_REQUIRE(path && out, "qma_cuda_model_load_gguf: bad arguments");
    Mapping f;
    int rc = f.open(path);
    if (rc) return rc;
    std::vector<qma_cuda_tensor> t;
    uint64_t off = 0;
    Hparams hp;
    if ((rc = parse(static_cast<const uint8_t *>(f.p), f.size, t, off, hp))) return rc;
    return qma_cuda_model_load(device, t.data(), uint32_t(t.size()), static_cast<const uint8_t *>(f.p) + off,
                               f.size - off, out);
}

}  // extern "C"
