// ckpt.cu -- routed experts from the checkpoint's safetensors shards into the HBM pool.
//
// Host side of the path (src/io/k3_st.c, src/io/k3_load.c in the reference): index the
// shards of a checkpoint directory, resolve one expert's six tensors (w1, w2, w3, each
// weight_packed and weight_scale) into a byte run, read that run -- one O_DIRECT read widened
// to 4 KB boundaries when the six tensors tile a contiguous span, six reads in the canonical
// order otherwise -- and upload it into a pool-format device run (copy to a device staging
// buffer, then the pool pack kernel of moe_pool.cu). The host memory the read fills is the
// caller's (page aligned for O_DIRECT; pinned if the upload should be asynchronous).
#include <cuda_runtime.h>
#include <dirent.h>
#include <errno.h>
#include <fcntl.h>
#include <stdio.h>
#include <string.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"

namespace k3c {

constexpr int64_t CK_ALIGN = 4096;              // O_DIRECT offset/length/address granularity
constexpr int64_t CK_READ_MAX = 1LL << 30;      // bytes per pread call

static int dtype_size(int dt) {
    switch (dt) {
    case K3C_DT_U8: return 1;
    case K3C_DT_BF16:
    case K3C_DT_F16: return 2;
    case K3C_DT_F32: return 4;
    default: return 0;
    }
}

// ------------------------------------------------------------------ header scanner
// The safetensors header is a JSON object: tensor name -> {"dtype": s, "shape": [ints],
// "data_offsets": [begin, end]}, plus an optional "__metadata__" entry. The scanner reads that
// shape of document and skips any other value (objects, arrays, strings, numbers, literals).
class HeaderScan {
  public:
    HeaderScan(const char *p, const char *e) : p_(p), e_(e) {}

    void space() {
        while (p_ < e_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) p_++;
    }
    bool eat(char c) {
        space();
        if (p_ < e_ && *p_ == c) {
            p_++;
            return true;
        }
        return false;
    }
    bool string(std::string &out) {
        if (!eat('"')) return false;
        out.clear();
        while (p_ < e_ && *p_ != '"') {
            char c = *p_++;
            if (c == '\\') {
                if (p_ >= e_) return false;
                const char esc = *p_++;
                switch (esc) {
                case 'n': c = '\n'; break;
                case 't': c = '\t'; break;
                case 'r': c = '\r'; break;
                case 'b': c = '\b'; break;
                case 'f': c = '\f'; break;
                case 'u': {
                    // names in this format are ASCII: an ASCII code point is kept, any other
                    // becomes '?' (the name still resolves, as the reference's index does)
                    if (e_ - p_ < 4) return false;
                    unsigned v = 0;
                    for (int i = 0; i < 4; i++) {
                        const char h = p_[i];
                        const int d = h >= '0' && h <= '9' ? h - '0' : h >= 'a' && h <= 'f' ? h - 'a' + 10
                                      : h >= 'A' && h <= 'F' ? h - 'A' + 10 : -1;
                        if (d < 0) return false;
                        v = v * 16 + (unsigned)d;
                    }
                    p_ += 4;
                    c = v < 0x80 ? (char)v : '?';
                    break;
                }
                default: c = esc; break;   // \" \\ \/
                }
            }
            out.push_back(c);
        }
        if (p_ >= e_) return false;
        p_++;   // closing quote
        return true;
    }
    bool integer(int64_t &v) {
        space();
        bool neg = false;
        if (p_ < e_ && *p_ == '-') {
            neg = true;
            p_++;
        }
        if (p_ >= e_ || *p_ < '0' || *p_ > '9') return false;
        int64_t a = 0;
        while (p_ < e_ && *p_ >= '0' && *p_ <= '9') {
            if (a > (INT64_MAX - 9) / 10) return false;
            a = a * 10 + (*p_++ - '0');
        }
        v = neg ? -a : a;
        return true;
    }
    bool skip(int depth = 0) {
        if (depth > 64) return false;
        space();
        if (p_ >= e_) return false;
        const char c = *p_;
        if (c == '"') {
            std::string tmp;
            return string(tmp);
        }
        if (c == '{' || c == '[') {
            const char close = c == '{' ? '}' : ']';
            p_++;
            if (eat(close)) return true;
            for (;;) {
                if (c == '{') {
                    std::string k;
                    if (!string(k) || !eat(':')) return false;
                }
                if (!skip(depth + 1)) return false;
                if (eat(',')) continue;
                return eat(close);
            }
        }
        // number or literal: up to the next delimiter
        const char *s = p_;
        while (p_ < e_ && !strchr(",}] \t\r\n", *p_)) p_++;
        return p_ > s;
    }
    long pos(const char *base) const { return (long)(p_ - base); }

  private:
    const char *p_, *e_;
};

}  // namespace k3c

struct k3c_ckpt {
    std::vector<std::string> path;
    std::vector<int> fd, dfd;   // per shard: buffered descriptor, O_DIRECT descriptor or -1
    std::vector<k3c_tensor> t;
    std::vector<std::string> name;
    std::unordered_map<std::string, int> index;
};

namespace k3c {

static int dtype_code(const std::string &s) {
    if (s == "U8") return K3C_DT_U8;
    if (s == "BF16") return K3C_DT_BF16;
    if (s == "F16") return K3C_DT_F16;
    if (s == "F32") return K3C_DT_F32;
    return 0;
}

// Index one shard into c. Errors name the file and what is wrong with it.
static int index_shard(k3c_ckpt *c, int shard, const std::string &path) {
    const int fd = open(path.c_str(), O_RDONLY);
    if (fd < 0) return set_error(K3C_EINVAL, "ckpt: cannot open %s: %s", path.c_str(), strerror(errno));
    c->fd[shard] = fd;
    unsigned char lb[8];
    if (pread(fd, lb, 8, 0) != 8) return set_error(K3C_EINVAL, "ckpt: %s is shorter than a header length", path.c_str());
    uint64_t hlen = 0;
    for (int i = 7; i >= 0; i--) hlen = hlen << 8 | lb[i];
    struct stat st;
    if (fstat(fd, &st) != 0) return set_error(K3C_EINVAL, "ckpt: cannot stat %s", path.c_str());
    const int64_t fsize = (int64_t)st.st_size;
    if (hlen == 0 || hlen > (uint64_t)fsize || (int64_t)hlen > fsize - 8)
        return set_error(K3C_EINVAL, "ckpt: %s: header length %llu does not fit a %lld-byte file", path.c_str(),
                         (unsigned long long)hlen, (long long)fsize);
    std::string json((size_t)hlen, '\0');
    for (uint64_t got = 0; got < hlen;) {
        const ssize_t r = pread(fd, &json[got], (size_t)(hlen - got), (off_t)(8 + got));
        if (r <= 0) return set_error(K3C_EINVAL, "ckpt: %s: short read of the header", path.c_str());
        got += (uint64_t)r;
    }
    const int64_t base = 8 + (int64_t)hlen;   // data_offsets count from here
    const char *b = json.data();
    HeaderScan sc(b, b + json.size());
    if (!sc.eat('{')) return set_error(K3C_EINVAL, "ckpt: %s: the header is not a JSON object", path.c_str());
    bool first = true;
    while (!sc.eat('}')) {
        if (!first && !sc.eat(',')) return set_error(K3C_EINVAL, "ckpt: %s: expected ',' at byte %ld", path.c_str(), sc.pos(b));
        first = false;
        if (sc.eat('}')) break;   // tolerate a trailing comma
        std::string nm;
        if (!sc.string(nm) || !sc.eat(':'))
            return set_error(K3C_EINVAL, "ckpt: %s: bad entry name at byte %ld", path.c_str(), sc.pos(b));
        if (nm == "__metadata__") {
            if (!sc.skip()) return set_error(K3C_EINVAL, "ckpt: %s: bad __metadata__", path.c_str());
            continue;
        }
        if (!sc.eat('{')) return set_error(K3C_EINVAL, "ckpt: %s: entry %s is not an object", path.c_str(), nm.c_str());
        k3c_tensor t;
        memset(&t, 0, sizeof t);
        t.shard = shard;
        bool got_dt = false, got_off = false, f1 = true;
        int64_t o0 = 0, o1 = 0;
        while (!sc.eat('}')) {
            if (!f1 && !sc.eat(',')) return set_error(K3C_EINVAL, "ckpt: %s: malformed entry %s", path.c_str(), nm.c_str());
            f1 = false;
            std::string key;
            if (!sc.string(key) || !sc.eat(':'))
                return set_error(K3C_EINVAL, "ckpt: %s: malformed entry %s", path.c_str(), nm.c_str());
            if (key == "dtype") {
                std::string dv;
                if (!sc.string(dv)) return set_error(K3C_EINVAL, "ckpt: %s: bad dtype on %s", path.c_str(), nm.c_str());
                t.dtype = dtype_code(dv);
                if (!t.dtype)
                    return set_error(K3C_EINVAL, "ckpt: %s: unsupported dtype '%s' on %s", path.c_str(), dv.c_str(),
                                     nm.c_str());
                got_dt = true;
            } else if (key == "shape") {
                if (!sc.eat('[')) return set_error(K3C_EINVAL, "ckpt: %s: bad shape on %s", path.c_str(), nm.c_str());
                if (!sc.eat(']')) {
                    for (;;) {
                        int64_t d;
                        if (!sc.integer(d) || d < 0)
                            return set_error(K3C_EINVAL, "ckpt: %s: bad shape on %s", path.c_str(), nm.c_str());
                        if (t.ndim == 4) return set_error(K3C_EINVAL, "ckpt: %s: %s has rank > 4", path.c_str(), nm.c_str());
                        t.shape[t.ndim++] = d;
                        if (sc.eat(',')) continue;
                        if (sc.eat(']')) break;
                        return set_error(K3C_EINVAL, "ckpt: %s: bad shape on %s", path.c_str(), nm.c_str());
                    }
                }
            } else if (key == "data_offsets") {
                if (!sc.eat('[') || !sc.integer(o0) || !sc.eat(',') || !sc.integer(o1) || !sc.eat(']'))
                    return set_error(K3C_EINVAL, "ckpt: %s: bad data_offsets on %s", path.c_str(), nm.c_str());
                got_off = true;
            } else if (!sc.skip()) {
                return set_error(K3C_EINVAL, "ckpt: %s: malformed entry %s", path.c_str(), nm.c_str());
            }
        }
        if (!got_dt || !got_off)
            return set_error(K3C_EINVAL, "ckpt: %s: %s lacks dtype or data_offsets", path.c_str(), nm.c_str());
        int64_t numel = 1;
        for (int i = 0; i < t.ndim; i++) numel *= t.shape[i];
        t.off = base + o0;
        t.nbytes = o1 - o0;
        // the span must be exactly the shape's bytes, or every later read of it is misaligned
        if (o0 < 0 || t.nbytes != numel * dtype_size(t.dtype))
            return set_error(K3C_EINVAL, "ckpt: %s: %s spans %lld bytes, its shape needs %lld", path.c_str(), nm.c_str(),
                             (long long)t.nbytes, (long long)(numel * dtype_size(t.dtype)));
        if (base + o1 > fsize) return set_error(K3C_EINVAL, "ckpt: %s: %s ends past the end of the file", path.c_str(), nm.c_str());
        if (!c->index.emplace(nm, (int)c->t.size()).second)
            return set_error(K3C_EINVAL, "ckpt: tensor %s appears twice", nm.c_str());
        c->t.push_back(t);
        c->name.push_back(nm);
    }
    // the page cache cannot help an expert read once per use: a second descriptor bypasses
    // it where the file system allows O_DIRECT (otherwise reads go through fd)
    c->dfd[shard] = open(path.c_str(), O_RDONLY | O_DIRECT);
    return K3C_OK;
}

// Widened O_DIRECT read of [off, off + n) into buf (page aligned, bufcap bytes); the payload
// starts at *pad. Without an O_DIRECT descriptor, or into a buffer that is not page aligned, a
// buffered read at buf + 0.
static int64_t read_fd_span(int fd, int dfd_in, int64_t off, int64_t n, void *buf, int64_t bufcap, int64_t *pad) {
    // O_DIRECT also needs the destination aligned: a buffer that is not takes the buffered path
    const int dfd = ((uintptr_t)buf % CK_ALIGN) ? -1 : dfd_in;
    if (dfd < 0) {
        if (pad) *pad = 0;
        if (bufcap < n) return 0;
        int64_t got = 0;
        while (got < n) {
            const int64_t want = std::min(n - got, CK_READ_MAX);
            const ssize_t r = pread(fd, (char *)buf + got, (size_t)want, (off_t)(off + got));
            if (r <= 0) break;
            got += r;
        }
        return got;
    }
    const int64_t lo = off / CK_ALIGN * CK_ALIGN;
    const int64_t hi = (off + n + CK_ALIGN - 1) / CK_ALIGN * CK_ALIGN;
    if (hi - lo > bufcap) return 0;
    if (pad) *pad = off - lo;
    int64_t got = 0;
    while (got < hi - lo) {
        const int64_t want = std::min(hi - lo - got, CK_READ_MAX);
        const ssize_t r = pread(dfd, (char *)buf + got, (size_t)want, (off_t)(lo + got));
        if (r <= 0) break;   // the last window may run past the end of the file
        got += r;
    }
    const int64_t pl = off - lo;
    return got >= pl + n ? n : (got > pl ? got - pl : 0);
}

static int64_t read_span(const k3c_ckpt *c, int shard, int64_t off, int64_t n, void *buf, int64_t bufcap,
                         int64_t *pad) {
    return read_fd_span(c->fd[shard], c->dfd[shard], off, n, buf, bufcap, pad);
}

}  // namespace k3c

using namespace k3c;

extern "C" k3c_ckpt *k3c_ckpt_open(const char *dir) {
    clear_error();
    if (!dir) {
        set_error(K3C_EINVAL, "ckpt_open: null directory");
        return nullptr;
    }
    DIR *d = opendir(dir);
    if (!d) {
        set_error(K3C_EINVAL, "ckpt_open: cannot open directory %s", dir);
        return nullptr;
    }
    std::vector<std::string> files;
    for (struct dirent *e; (e = readdir(d)) != nullptr;) {
        const std::string n = e->d_name;
        if (n.size() > 12 && n.compare(n.size() - 12, 12, ".safetensors") == 0) files.push_back(n);
    }
    closedir(d);
    if (files.empty()) {
        set_error(K3C_ENOTFOUND, "ckpt_open: no .safetensors files in %s", dir);
        return nullptr;
    }
    std::sort(files.begin(), files.end());   // shard numbers do not depend on directory order
    k3c_ckpt *c = new k3c_ckpt;
    c->fd.assign(files.size(), -1);
    c->dfd.assign(files.size(), -1);
    for (size_t i = 0; i < files.size(); i++) {
        c->path.push_back(std::string(dir) + "/" + files[i]);
        if (index_shard(c, (int)i, c->path.back()) != K3C_OK) {
            const std::string msg = k3c_last_error();
            k3c_ckpt_close(c);
            set_error(K3C_EINVAL, "%s", msg.c_str());
            return nullptr;
        }
    }
    return c;
}

extern "C" void k3c_ckpt_close(k3c_ckpt *c) {
    if (!c) return;
    for (int fd : c->fd)
        if (fd >= 0) close(fd);
    for (int fd : c->dfd)
        if (fd >= 0) close(fd);
    delete c;
}

extern "C" int k3c_ckpt_shards(const k3c_ckpt *c) { return c ? (int)c->path.size() : 0; }

extern "C" int k3c_ckpt_direct(const k3c_ckpt *c, int shard) {
    return c && shard >= 0 && shard < (int)c->dfd.size() && c->dfd[shard] >= 0;
}

extern "C" int k3c_ckpt_find(const k3c_ckpt *c, const char *name, k3c_tensor *t) {
    clear_error();
    if (!c || !name || !t) return set_error(K3C_EINVAL, "ckpt_find: bad arguments");
    const auto it = c->index.find(name);
    if (it == c->index.end()) return set_error(K3C_ENOTFOUND, "ckpt_find: no tensor %s", name);
    *t = c->t[it->second];
    return K3C_OK;
}

extern "C" int k3c_expert_ref(const k3c_ckpt *c, int layer, int expert, k3c_expert_run *r) {
    clear_error();
    if (!c || !r) return set_error(K3C_EINVAL, "expert_ref: bad arguments");
    memset(r, 0, sizeof *r);
    r->layer = layer;
    r->expert = expert;
    static const char *const mat[3] = {"w1", "w2", "w3"};
    k3c_tensor pk[3], sc[3];
    char nm[256];
    for (int i = 0; i < 3; i++) {
        for (int j = 0; j < 2; j++) {
            snprintf(nm, sizeof nm, "language_model.model.layers.%d.block_sparse_moe.experts.%d.%s.%s", layer, expert,
                     mat[i], j ? "weight_scale" : "weight_packed");
            const auto it = c->index.find(nm);
            if (it == c->index.end()) return set_error(K3C_ENOTFOUND, "expert_ref: missing %s", nm);
            (j ? sc : pk)[i] = c->t[it->second];
        }
        const k3c_tensor &p = pk[i], &s = sc[i];
        if (p.dtype != K3C_DT_U8 || s.dtype != K3C_DT_U8)
            return set_error(K3C_EINVAL, "expert_ref: layer %d expert %d %s is not U8", layer, expert, mat[i]);
        if (p.ndim != 2 || s.ndim != 2)
            return set_error(K3C_EINVAL, "expert_ref: layer %d expert %d %s is not 2-D", layer, expert, mat[i]);
        if (p.shape[0] != s.shape[0])
            return set_error(K3C_EINVAL, "expert_ref: layer %d expert %d %s: %lld packed rows, %lld scale rows", layer,
                             expert, mat[i], (long long)p.shape[0], (long long)s.shape[0]);
        // one E8M0 scale per 32 elements: any other count would apply scales to the wrong weights
        if (s.shape[1] * 32 != p.shape[1] * 2)
            return set_error(K3C_EINVAL, "expert_ref: layer %d expert %d %s: %lld scales for %lld elements is not a "
                             "group of 32", layer, expert, mat[i], (long long)s.shape[1], (long long)(p.shape[1] * 2));
        if (p.shard != s.shard || p.shard != pk[0].shard)
            return set_error(K3C_EINVAL, "expert_ref: layer %d expert %d spans shards", layer, expert);
        r->m[i].rows = (int)p.shape[0];
        r->m[i].pcols = (int)p.shape[1];
        r->m[i].scols = (int)s.shape[1];
        r->m[i].p_bytes = p.nbytes;
        r->m[i].s_bytes = s.nbytes;
    }
    r->shard = pk[0].shard;
    const k3c_tensor *six[6] = {&pk[0], &sc[0], &pk[1], &sc[1], &pk[2], &sc[2]};
    int64_t lo = six[0]->off, hi = 0, sum = 0;
    for (const k3c_tensor *t : six) {
        lo = std::min(lo, t->off);
        hi = std::max(hi, t->off + t->nbytes);
        sum += t->nbytes;
    }
    // contiguous when the six spans exactly tile [lo, hi); offsets then stay where the file has
    // them, otherwise the run is assembled in the order w1.packed w1.scale w2.packed ...
    r->contiguous = hi - lo == sum;
    r->off = lo;
    int64_t o = 0;
    for (int i = 0; i < 3; i++) {
        if (r->contiguous) {
            r->m[i].p_off = pk[i].off - lo;
            r->m[i].s_off = sc[i].off - lo;
        } else {
            r->m[i].p_off = o;
            o += r->m[i].p_bytes;
            r->m[i].s_off = o;
            o += r->m[i].s_bytes;
        }
    }
    r->nbytes = r->contiguous ? sum : o;
    return K3C_OK;
}

extern "C" int64_t k3c_expert_read(const k3c_ckpt *c, const k3c_expert_run *r, void *buf, int64_t bufcap,
                                   int64_t *payload_off) {
    clear_error();
    if (!c || !r || !buf || r->shard < 0 || r->shard >= (int)c->path.size()) {
        set_error(K3C_EINVAL, "expert_read: bad arguments");
        return 0;
    }
    if (r->contiguous) {
        const int64_t n = read_span(c, r->shard, r->off, r->nbytes, buf, bufcap, payload_off);
        if (n != r->nbytes) set_error(K3C_EINVAL, "expert_read: read %lld of %lld bytes", (long long)n, (long long)r->nbytes);
        return n;
    }
    // scattered tensors: one buffered read each, into the canonical order
    if (payload_off) *payload_off = 0;
    if (bufcap < r->nbytes) {
        set_error(K3C_EINVAL, "expert_read: buffer of %lld bytes for a %lld-byte run", (long long)bufcap, (long long)r->nbytes);
        return 0;
    }
    static const char *const mat[3] = {"w1", "w2", "w3"};
    char nm[256];
    int64_t got = 0;
    for (int i = 0; i < 3; i++) {
        for (int j = 0; j < 2; j++) {
            snprintf(nm, sizeof nm, "language_model.model.layers.%d.block_sparse_moe.experts.%d.%s.%s", r->layer,
                     r->expert, mat[i], j ? "weight_scale" : "weight_packed");
            const auto it = c->index.find(nm);
            if (it == c->index.end()) {
                set_error(K3C_ENOTFOUND, "expert_read: missing %s", nm);
                return got;
            }
            const k3c_tensor &t = c->t[it->second];
            char *dst = (char *)buf + (j ? r->m[i].s_off : r->m[i].p_off);
            int64_t n = 0;
            while (n < t.nbytes) {
                const ssize_t q = pread(c->fd[t.shard], dst + n, (size_t)std::min(t.nbytes - n, CK_READ_MAX),
                                        (off_t)(t.off + n));
                if (q <= 0) break;
                n += q;
            }
            got += n;
        }
    }
    if (got != r->nbytes) set_error(K3C_EINVAL, "expert_read: read %lld of %lld bytes", (long long)got, (long long)r->nbytes);
    return got;
}

extern "C" int k3c_expert_upload(uint8_t *dev_run, const k3c_expert_run *r, const void *payload, uint8_t *dev_staging,
                                 k3c_stream_t stream) {
    clear_error();
    if (!dev_run || !r || !payload || !dev_staging) return set_error(K3C_EINVAL, "expert_upload: bad arguments");
    // w1 (gate) and w3 (up) are [inter][hidden/2]; w2 (down) is [hidden][inter/2]
    const int inter = r->m[0].rows, hidden = 2 * r->m[0].pcols;
    if (r->m[2].rows != inter || r->m[2].pcols != r->m[0].pcols || r->m[1].rows != hidden ||
        2 * r->m[1].pcols != inter)
        return set_error(K3C_EINVAL, "expert_upload: w1 %dx%d, w2 %dx%d, w3 %dx%d are not one expert's shapes",
                         r->m[0].rows, 2 * r->m[0].pcols, r->m[1].rows, 2 * r->m[1].pcols, r->m[2].rows,
                         2 * r->m[2].pcols);
    cudaStream_t s = (cudaStream_t)stream;
    K3C_TRY_CUDA(cudaMemcpyAsync(dev_staging, payload, (size_t)r->nbytes, cudaMemcpyHostToDevice, s));
    K3ExpertQ q;
    q.p1 = dev_staging + r->m[0].p_off;
    q.s1 = dev_staging + r->m[0].s_off;
    q.p3 = dev_staging + r->m[2].p_off;
    q.s3 = dev_staging + r->m[2].s_off;
    q.p2 = dev_staging + r->m[1].p_off;
    q.s2 = dev_staging + r->m[1].s_off;
    return k3c_pool_pack_expert(dev_run, &q, hidden, inter, stream);
}

// ------------------------------------------------------------------ packed trunk
// trunk.json: {"align": 4096, "layers": [{"file_off": F, "nbytes": N, "tensors": {name: {"off": o,
// "nbytes": n, "dtype": "BF16" | "F32" | "U8" | "F16" | "I8R", "shape": [...]}}, ...}, ...]}
// (src/io/k3_trunk.c:98-148; other keys are skipped as there).
struct k3c_trunk {
    int fd = -1, dfd = -1;
    int64_t align = 0;
    struct Layer {
        int64_t file_off = 0, nbytes = 0;
        std::unordered_map<std::string, k3c_tensor> t;
    };
    std::vector<Layer> lay;
};

namespace k3c {

static int trunk_dtype(const std::string &s) {
    if (s == "I8R") return K3C_DT_I8R;
    return dtype_code(s);
}

static int parse_trunk_tensor(HeaderScan &sc, k3c_tensor &t, const std::string &nm) {
    memset(&t, 0, sizeof t);
    if (!sc.eat('{')) return set_error(K3C_EINVAL, "trunk: tensor %s is not an object", nm.c_str());
    bool f1 = true, got_dt = false;
    while (!sc.eat('}')) {
        if (!f1 && !sc.eat(',')) return set_error(K3C_EINVAL, "trunk: malformed tensor %s", nm.c_str());
        f1 = false;
        std::string key;
        if (!sc.string(key) || !sc.eat(':')) return set_error(K3C_EINVAL, "trunk: malformed tensor %s", nm.c_str());
        if (key == "off" || key == "nbytes") {
            int64_t v;
            if (!sc.integer(v) || v < 0) return set_error(K3C_EINVAL, "trunk: bad %s on %s", key.c_str(), nm.c_str());
            (key == "off" ? t.off : t.nbytes) = v;
        } else if (key == "dtype") {
            std::string dv;
            if (!sc.string(dv)) return set_error(K3C_EINVAL, "trunk: bad dtype on %s", nm.c_str());
            t.dtype = trunk_dtype(dv);
            if (!t.dtype) return set_error(K3C_EINVAL, "trunk: unsupported dtype '%s' on %s", dv.c_str(), nm.c_str());
            got_dt = true;
        } else if (key == "shape") {
            if (!sc.eat('[')) return set_error(K3C_EINVAL, "trunk: bad shape on %s", nm.c_str());
            if (!sc.eat(']'))
                for (;;) {
                    int64_t d;
                    if (!sc.integer(d) || d < 0 || t.ndim == 4)
                        return set_error(K3C_EINVAL, "trunk: bad shape on %s", nm.c_str());
                    t.shape[t.ndim++] = d;
                    if (sc.eat(',')) continue;
                    if (sc.eat(']')) break;
                    return set_error(K3C_EINVAL, "trunk: bad shape on %s", nm.c_str());
                }
        } else if (!sc.skip()) {
            return set_error(K3C_EINVAL, "trunk: malformed tensor %s", nm.c_str());
        }
    }
    if (!got_dt) return set_error(K3C_EINVAL, "trunk: %s has no dtype", nm.c_str());
    // the span must be the shape's bytes; an I8R matrix is rows x (4-byte scale + cols int8)
    int64_t want;
    if (t.dtype == K3C_DT_I8R) {
        if (t.ndim != 2) return set_error(K3C_EINVAL, "trunk: I8R tensor %s is not 2-D", nm.c_str());
        want = t.shape[0] * (4 + t.shape[1]);
    } else {
        want = dtype_size(t.dtype);
        for (int i = 0; i < t.ndim; i++) want *= t.shape[i];
    }
    if (t.nbytes != want)
        return set_error(K3C_EINVAL, "trunk: %s spans %lld bytes, its shape needs %lld", nm.c_str(),
                         (long long)t.nbytes, (long long)want);
    return K3C_OK;
}

static int parse_trunk(k3c_trunk *tr, const std::string &txt) {
    HeaderScan sc(txt.data(), txt.data() + txt.size());
    if (!sc.eat('{')) return set_error(K3C_EINVAL, "trunk: trunk.json is not an object");
    bool f1 = true, got_layers = false;
    while (!sc.eat('}')) {
        if (!f1 && !sc.eat(',')) return set_error(K3C_EINVAL, "trunk: malformed trunk.json");
        f1 = false;
        std::string key;
        if (!sc.string(key) || !sc.eat(':')) return set_error(K3C_EINVAL, "trunk: malformed trunk.json");
        if (key == "align") {
            if (!sc.integer(tr->align)) return set_error(K3C_EINVAL, "trunk: bad align");
        } else if (key == "layers") {
            got_layers = true;
            if (!sc.eat('[')) return set_error(K3C_EINVAL, "trunk: layers is not an array");
            if (sc.eat(']')) continue;
            for (;;) {
                k3c_trunk::Layer L;
                if (!sc.eat('{')) return set_error(K3C_EINVAL, "trunk: layer %zu is not an object", tr->lay.size());
                bool g1 = true, got_t = false;
                while (!sc.eat('}')) {
                    if (!g1 && !sc.eat(',')) return set_error(K3C_EINVAL, "trunk: malformed layer %zu", tr->lay.size());
                    g1 = false;
                    std::string lk;
                    if (!sc.string(lk) || !sc.eat(':'))
                        return set_error(K3C_EINVAL, "trunk: malformed layer %zu", tr->lay.size());
                    if (lk == "file_off" || lk == "nbytes") {
                        int64_t v;
                        if (!sc.integer(v) || v < 0) return set_error(K3C_EINVAL, "trunk: bad %s", lk.c_str());
                        (lk == "file_off" ? L.file_off : L.nbytes) = v;
                    } else if (lk == "tensors") {
                        got_t = true;
                        if (!sc.eat('{')) return set_error(K3C_EINVAL, "trunk: layer %zu tensors", tr->lay.size());
                        bool h1 = true;
                        while (!sc.eat('}')) {
                            if (!h1 && !sc.eat(',')) return set_error(K3C_EINVAL, "trunk: malformed tensors");
                            h1 = false;
                            std::string nm;
                            if (!sc.string(nm) || !sc.eat(':')) return set_error(K3C_EINVAL, "trunk: malformed tensors");
                            k3c_tensor t;
                            K3C_TRY(parse_trunk_tensor(sc, t, nm));
                            if (!L.t.emplace(nm, t).second)
                                return set_error(K3C_EINVAL, "trunk: %s appears twice in layer %zu", nm.c_str(),
                                                 tr->lay.size());
                        }
                    } else if (!sc.skip()) {
                        return set_error(K3C_EINVAL, "trunk: malformed layer %zu", tr->lay.size());
                    }
                }
                if (!got_t) return set_error(K3C_EINVAL, "trunk: layer %zu has no tensors", tr->lay.size());
                for (auto &kv : L.t)
                    if (kv.second.off + kv.second.nbytes > L.nbytes)
                        return set_error(K3C_EINVAL, "trunk: %s runs past its layer's %lld bytes", kv.first.c_str(),
                                         (long long)L.nbytes);
                tr->lay.push_back(std::move(L));
                if (sc.eat(',')) continue;
                if (sc.eat(']')) break;
                return set_error(K3C_EINVAL, "trunk: malformed layers array");
            }
        } else if (!sc.skip()) {
            return set_error(K3C_EINVAL, "trunk: malformed trunk.json");
        }
    }
    if (!got_layers) return set_error(K3C_EINVAL, "trunk: no layers array");
    return K3C_OK;
}

}  // namespace k3c

extern "C" void k3c_trunk_close(k3c_trunk *tr) {
    if (!tr) return;
    if (tr->fd >= 0) close(tr->fd);
    if (tr->dfd >= 0) close(tr->dfd);
    delete tr;
}

extern "C" k3c_trunk *k3c_trunk_open(const char *dir) {
    clear_error();
    if (!dir) {
        set_error(K3C_EINVAL, "trunk_open: null directory");
        return nullptr;
    }
    const std::string jp = std::string(dir) + "/trunk.json", bp = std::string(dir) + "/trunk.bin";
    FILE *f = fopen(jp.c_str(), "rb");
    if (!f) {
        set_error(K3C_EINVAL, "trunk_open: cannot read %s", jp.c_str());
        return nullptr;
    }
    std::string txt;
    char chunk[65536];
    for (size_t n; (n = fread(chunk, 1, sizeof chunk, f)) > 0;) txt.append(chunk, n);
    fclose(f);
    k3c_trunk *tr = new k3c_trunk;
    if (parse_trunk(tr, txt) != K3C_OK) {
        k3c_trunk_close(tr);
        return nullptr;
    }
    tr->fd = open(bp.c_str(), O_RDONLY);
    if (tr->fd < 0) {
        set_error(K3C_EINVAL, "trunk_open: cannot open %s", bp.c_str());
        k3c_trunk_close(tr);
        return nullptr;
    }
    struct stat st;
    const int64_t fsize = fstat(tr->fd, &st) == 0 ? (int64_t)st.st_size : -1;
    for (size_t i = 0; i < tr->lay.size(); i++)
        if (tr->lay[i].file_off + tr->lay[i].nbytes > fsize) {
            set_error(K3C_EINVAL, "trunk_open: layer %zu runs past the end of %s", i, bp.c_str());
            k3c_trunk_close(tr);
            return nullptr;
        }
    // O_DIRECT only for a trunk packed on 4096-byte boundaries (k3_trunk_open's rule)
    if (tr->align == CK_ALIGN) tr->dfd = open(bp.c_str(), O_RDONLY | O_DIRECT);
    return tr;
}

extern "C" int k3c_trunk_layers(const k3c_trunk *tr) { return tr ? (int)tr->lay.size() : 0; }

extern "C" int k3c_trunk_find(const k3c_trunk *tr, int layer, const char *name, k3c_tensor *t) {
    clear_error();
    if (!tr || !name || !t || layer < 0 || layer >= (int)tr->lay.size())
        return set_error(K3C_EINVAL, "trunk_find: bad arguments (layer %d)", layer);
    const auto &L = tr->lay[(size_t)layer];
    auto it = L.t.find(name);
    if (it == L.t.end()) return set_error(K3C_ENOTFOUND, "trunk_find: %s not in layer %d", name, layer);
    *t = it->second;
    t->off += L.file_off;
    t->shard = 0;
    return K3C_OK;
}

extern "C" int64_t k3c_trunk_read(const k3c_trunk *tr, const k3c_tensor *t, void *buf, int64_t bufcap,
                                  int64_t *payload_off) {
    clear_error();
    if (!tr || !t || !buf || bufcap <= 0) return set_error(K3C_EINVAL, "trunk_read: bad arguments");
    int64_t pad = 0;
    const int64_t got = read_fd_span(tr->fd, tr->dfd, t->off, t->nbytes, buf, bufcap, &pad);
    if (payload_off) *payload_off = pad;
    if (got != t->nbytes)
        set_error(K3C_EINVAL, "trunk_read: read %lld of %lld bytes", (long long)got, (long long)t->nbytes);
    return got;
}
