// pool.cu -- HBM expert pool: the reference's expert cache (src/cache/k3_cache.c:24-261,
// K3ExpertSrc get/getmany/resident, include/k3/k3.h:318-355) rebuilt for a GPU whose experts
// stream from pinned host memory instead of disk.
//
// Same bookkeeping as the reference: one slot per resident expert, key = layer*n_experts +
// expert, slot states key / EMPTY / INFLIGHT, victim = an EMPTY slot if any, else the least
// recently used slot that is neither pinned nor in flight (pick_victim, k3_cache.c:46-57);
// hits, misses, evictions and batch-prefetch reads counted the reference's way, including its
// "true resident hit rate" (hits minus prefetch reads, k3_cache.c:416-425).
//
// What changes on the GPU: a miss becomes one cudaMemcpyAsync of the expert's pool-format
// run from pinned host memory into its slot on the pool's own copy stream, so copies overlap
// kernels. Instead of the reference's synchronous read, every slot carries two events:
//   fill   recorded on the copy stream after the slot's copy; a consumer's stream waits on
//          it before reading the slot (the INFLIGHT state of the reference lasts until then);
//   use    recorded on the consumer's stream when it releases the slot; the copy stream
//          waits on it before overwriting the slot with another expert.
// A slot is pinned from acquire to release, so the experts of a layer in flight cannot be
// evicted under it (the reference's "pointers stay valid until the token finishes").
#include <cuda_runtime.h>
#include <stdio.h>

#include <mutex>
#include <utility>
#include <vector>

#include "common.cuh"
#include "pool_common.cuh"

struct k3c_expert_pool {
    int hidden = 0, inter = 0, n_layers = 0, n_experts = 0, nslot = 0;
    size_t stride = 0, run_bytes = 0;
    uint8_t *arena = nullptr;
    cudaStream_t copy = nullptr;
    k3c_pool_src_fn src = nullptr;
    void *src_ctx = nullptr;
    std::vector<int> slot_of;       // key -> slot or -1
    std::vector<int> key_of;        // slot -> key, K3C_SLOT_EMPTY or K3C_SLOT_INFLIGHT
    std::vector<int> pins;          // acquire count + permanent pins
    std::vector<char> pinned_forever;
    std::vector<char> user_pin;     // k3c_pool_set_pin (the reference's k3_cache_pin)
    std::vector<int32_t> trace;     // (layer, expert) of every get request, in order
    std::vector<uint32_t> hist;     // get requests per key
    std::vector<unsigned long long> used_at;
    std::vector<cudaEvent_t> fill_ev, use_ev;
    std::vector<char> fill_pending, use_pending;
    unsigned long long clock = 0;
    k3c_pool_stats_t st{};
    // pinned staging for the run_of tables handed to the kernels
    std::vector<int *> stage;
    std::vector<cudaEvent_t> stage_ev;
    int stage_next = 0;
    std::mutex mu;
};

namespace {

constexpr int kStageRing = 64;

int pick_victim(k3c_expert_pool *p) {
    int best = -1;
    unsigned long long oldest = ~0ull;
    for (int i = 0; i < p->nslot; i++) {
        if (p->key_of[i] == K3C_SLOT_INFLIGHT) continue;
        if (p->key_of[i] == K3C_SLOT_EMPTY) return i;
        if (p->pins[i] > 0 || p->user_pin[i]) continue;
        if (p->used_at[i] < oldest) {
            oldest = p->used_at[i];
            best = i;
        }
    }
    return best;
}

// Copies key's run into a victim slot and publishes it. Returns the slot or a negative
// status (the slot is left EMPTY when the copy could not be issued).
int fill(k3c_expert_pool *p, int layer, int expert) {
    const int key = layer * p->n_experts + expert;
    const void *host = p->src ? p->src(p->src_ctx, layer, expert) : nullptr;
    if (!host) return k3c::set_error(K3C_ENOTFOUND, "pool: no host bytes for layer %d expert %d", layer, expert);
    const int slot = pick_victim(p);
    if (slot < 0) return k3c::set_error(K3C_EFULL, "pool: every slot is pinned or in flight");
    if (p->key_of[slot] >= 0) {
        p->slot_of[p->key_of[slot]] = -1;
        p->st.evictions++;
    }
    p->key_of[slot] = K3C_SLOT_INFLIGHT;
    if (p->use_pending[slot]) {   // the last consumer of the old expert must be done
        cudaError_t e = cudaStreamWaitEvent(p->copy, p->use_ev[slot], 0);
        if (e != cudaSuccess) {
            p->key_of[slot] = K3C_SLOT_EMPTY;
            return k3c::set_error(K3C_ECUDA, "pool: %s", cudaGetErrorString(e));
        }
    }
    cudaError_t e = cudaMemcpyAsync(p->arena + (size_t)slot * p->stride, host, p->run_bytes,
                                    cudaMemcpyHostToDevice, p->copy);
    if (e == cudaSuccess) e = cudaEventRecord(p->fill_ev[slot], p->copy);
    if (e != cudaSuccess) {
        p->key_of[slot] = K3C_SLOT_EMPTY;   // publish only what was issued
        return k3c::set_error(K3C_ECUDA, "pool: copy of layer %d expert %d: %s", layer, expert,
                              cudaGetErrorString(e));
    }
    p->fill_pending[slot] = 1;
    p->key_of[slot] = key;
    p->slot_of[key] = slot;
    p->used_at[slot] = ++p->clock;
    p->st.bytes_h2d += (long long)p->run_bytes;
    return slot;
}

bool key_ok(const k3c_expert_pool *p, int layer, int expert) {
    return layer >= 0 && layer < p->n_layers && expert >= 0 && expert < p->n_experts;
}

}  // namespace

extern "C" {

k3c_expert_pool *k3c_pool_create(int hidden, int inter, int n_layers, int n_experts, int n_slots,
                                 k3c_pool_src_fn src, void *ctx) {
    k3c::clear_error();
    const size_t run = k3c_pool_run_bytes(hidden, inter);
    if (!run || n_layers <= 0 || n_experts <= 0 || n_slots <= 0) {
        k3c::set_error(K3C_EINVAL, "pool: hidden=%d inter=%d layers=%d experts=%d slots=%d", hidden, inter,
                       n_layers, n_experts, n_slots);
        return nullptr;
    }
    k3c_expert_pool *p = new k3c_expert_pool;
    p->hidden = hidden;
    p->inter = inter;
    p->n_layers = n_layers;
    p->n_experts = n_experts;
    p->nslot = n_slots;
    p->run_bytes = run;
    p->stride = k3c::align_up(run, 256);
    p->src = src;
    p->src_ctx = ctx;
    bool ok = cudaMalloc((void **)&p->arena, p->stride * (size_t)n_slots) == cudaSuccess;
    ok = ok && cudaStreamCreateWithFlags(&p->copy, cudaStreamNonBlocking) == cudaSuccess;
    p->slot_of.assign((size_t)n_layers * n_experts, -1);
    p->key_of.assign(n_slots, K3C_SLOT_EMPTY);
    p->pins.assign(n_slots, 0);
    p->pinned_forever.assign(n_slots, 0);
    p->user_pin.assign(n_slots, 0);
    p->hist.assign((size_t)n_layers * n_experts, 0);
    p->used_at.assign(n_slots, 0);
    p->fill_ev.assign(n_slots, nullptr);
    p->use_ev.assign(n_slots, nullptr);
    p->fill_pending.assign(n_slots, 0);
    p->use_pending.assign(n_slots, 0);
    for (int i = 0; ok && i < n_slots; i++)
        ok = cudaEventCreateWithFlags(&p->fill_ev[i], cudaEventDisableTiming) == cudaSuccess &&
             cudaEventCreateWithFlags(&p->use_ev[i], cudaEventDisableTiming) == cudaSuccess;
    p->stage.assign(kStageRing, nullptr);
    p->stage_ev.assign(kStageRing, nullptr);
    for (int i = 0; ok && i < kStageRing; i++)
        ok = cudaMallocHost((void **)&p->stage[i], (size_t)n_experts * sizeof(int)) == cudaSuccess &&
             cudaEventCreateWithFlags(&p->stage_ev[i], cudaEventDisableTiming) == cudaSuccess;
    if (!ok) {
        k3c::set_error(K3C_ENOMEM, "pool: cannot allocate %d slots of %zu bytes", n_slots, p->stride);
        k3c_pool_destroy(p);
        cudaGetLastError();
        return nullptr;
    }
    return p;
}

void k3c_pool_destroy(k3c_expert_pool *p) {
    if (!p) return;
    if (p->copy) cudaStreamSynchronize(p->copy);
    for (cudaEvent_t e : p->fill_ev) if (e) cudaEventDestroy(e);
    for (cudaEvent_t e : p->use_ev) if (e) {
        cudaEventSynchronize(e);
        cudaEventDestroy(e);
    }
    for (size_t i = 0; i < p->stage.size(); i++) {
        if (p->stage_ev[i]) {
            cudaEventSynchronize(p->stage_ev[i]);
            cudaEventDestroy(p->stage_ev[i]);
        }
        if (p->stage[i]) cudaFreeHost(p->stage[i]);
    }
    if (p->copy) cudaStreamDestroy(p->copy);
    if (p->arena) cudaFree(p->arena);
    delete p;
}

uint8_t *k3c_pool_arena(k3c_expert_pool *p) { return p ? p->arena : nullptr; }
size_t k3c_pool_slot_stride(const k3c_expert_pool *p) { return p ? p->stride : 0; }
int k3c_pool_slots(const k3c_expert_pool *p) { return p ? p->nslot : 0; }

int k3c_pool_shape(const k3c_expert_pool *p, int *hidden, int *inter) {
    if (!p) return K3C_EINVAL;
    if (hidden) *hidden = p->hidden;
    if (inter) *inter = p->inter;
    return K3C_OK;
}

int k3c_pool_resident(k3c_expert_pool *p, int layer, int expert) {
    if (!p || !key_ok(p, layer, expert)) return -1;
    std::lock_guard<std::mutex> lk(p->mu);
    return p->slot_of[layer * p->n_experts + expert];
}

int k3c_pool_getmany(k3c_expert_pool *p, int layer, const int *ids, int n) {
    k3c::clear_error();
    if (!p || (n > 0 && !ids)) return k3c::set_error(K3C_EINVAL, "pool_getmany: null argument");
    std::lock_guard<std::mutex> lk(p->mu);
    int issued = 0;
    for (int i = 0; i < n; i++) {
        if (!key_ok(p, layer, ids[i])) continue;
        if (p->slot_of[layer * p->n_experts + ids[i]] >= 0) continue;   // resident or filling
        const int s = fill(p, layer, ids[i]);
        if (s == K3C_EFULL) break;
        if (s < 0) continue;   // this expert stays a miss for the get that follows
        p->st.prefetch_reads++;
        issued++;
    }
    return issued;
}

int k3c_pool_acquire(k3c_expert_pool *p, int layer, const int *ids, int n, int *slots, int *dev_run_of,
                     k3c_stream_t stream) {
    k3c::clear_error();
    if (!p || (n > 0 && !ids)) return k3c::set_error(K3C_EINVAL, "pool_acquire: null argument");
    cudaStream_t s = (cudaStream_t)stream;
    std::lock_guard<std::mutex> lk(p->mu);
    std::vector<int> got(n, -1);
    int rc = K3C_OK;
    for (int i = 0; i < n && rc == K3C_OK; i++) {
        if (!key_ok(p, layer, ids[i])) {
            rc = k3c::set_error(K3C_EINVAL, "pool_acquire: layer %d expert %d out of range", layer, ids[i]);
            break;
        }
        const int key = layer * p->n_experts + ids[i];
        p->hist[key]++;   // what was asked for, before it is served (k3_cache.c:235-249)
        p->trace.push_back(layer);
        p->trace.push_back(ids[i]);
        int slot = p->slot_of[key];
        if (slot >= 0) {
            p->st.hits++;
            p->used_at[slot] = ++p->clock;
        } else {
            p->st.misses++;
            slot = fill(p, layer, ids[i]);
            if (slot < 0) {
                rc = slot;
                break;
            }
        }
        p->pins[slot]++;
        got[i] = slot;
        if (p->fill_pending[slot]) {
            if (cudaEventQuery(p->fill_ev[slot]) == cudaSuccess) {
                p->fill_pending[slot] = 0;
            } else {
                cudaError_t e = cudaStreamWaitEvent(s, p->fill_ev[slot], 0);
                if (e != cudaSuccess) rc = k3c::set_error(K3C_ECUDA, "pool_acquire: %s", cudaGetErrorString(e));
            }
        }
    }
    cudaGetLastError();   // a not-ready event query is not an error
    if (rc != K3C_OK) {   // undo the pins taken so far
        for (int i = 0; i < n; i++)
            if (got[i] >= 0) p->pins[got[i]]--;
        return rc;
    }
    if (slots)
        for (int i = 0; i < n; i++) slots[i] = got[i];
    if (dev_run_of) {
        const int b = p->stage_next;
        p->stage_next = (b + 1) % kStageRing;
        cudaEventSynchronize(p->stage_ev[b]);   // the copy that last read this buffer is done
        int *h = p->stage[b];
        for (int e = 0; e < p->n_experts; e++) h[e] = -1;
        for (int i = 0; i < n; i++) h[ids[i]] = got[i];
        cudaError_t e = cudaMemcpyAsync(dev_run_of, h, (size_t)p->n_experts * sizeof(int), cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess) e = cudaEventRecord(p->stage_ev[b], s);
        if (e != cudaSuccess) return k3c::set_error(K3C_ECUDA, "pool_acquire: %s", cudaGetErrorString(e));
    }
    return K3C_OK;
}

int k3c_pool_release(k3c_expert_pool *p, int layer, const int *ids, int n, k3c_stream_t stream) {
    k3c::clear_error();
    if (!p || (n > 0 && !ids)) return k3c::set_error(K3C_EINVAL, "pool_release: null argument");
    std::lock_guard<std::mutex> lk(p->mu);
    for (int i = 0; i < n; i++) {
        if (!key_ok(p, layer, ids[i])) continue;
        const int slot = p->slot_of[layer * p->n_experts + ids[i]];
        if (slot < 0 || p->pins[slot] <= 0) continue;
        p->pins[slot]--;
        cudaError_t e = cudaEventRecord(p->use_ev[slot], (cudaStream_t)stream);
        if (e != cudaSuccess) return k3c::set_error(K3C_ECUDA, "pool_release: %s", cudaGetErrorString(e));
        p->use_pending[slot] = 1;
    }
    return K3C_OK;
}

int k3c_pool_pin(k3c_expert_pool *p, int layer, int expert, k3c_stream_t stream) {
    k3c::clear_error();
    if (!p || !key_ok(p, layer, expert)) return k3c::set_error(K3C_EINVAL, "pool_pin: bad key");
    int slot = -1;
    const int rc = k3c_pool_acquire(p, layer, &expert, 1, &slot, nullptr, stream);
    if (rc != K3C_OK) return rc;
    std::lock_guard<std::mutex> lk(p->mu);
    p->pinned_forever[slot] = 1;   // the acquire's pin is never released
    return slot;
}

int k3c_pool_stats(k3c_expert_pool *p, k3c_pool_stats_t *out) {
    if (!p || !out) return K3C_EINVAL;
    std::lock_guard<std::mutex> lk(p->mu);
    *out = p->st;
    return K3C_OK;
}

int k3c_pool_sync(k3c_expert_pool *p) {
    if (!p) return K3C_EINVAL;
    return cudaStreamSynchronize(p->copy) == cudaSuccess ? K3C_OK : K3C_ECUDA;
}

int k3c_pool_acquire_resident(k3c_expert_pool *p, int layer, int *ids, int cap, int *dev_run_of,
                              k3c_stream_t stream) {
    k3c::clear_error();
    if (!p || layer < 0 || layer >= p->n_layers) return k3c::set_error(K3C_EINVAL, "pool_acquire_resident: bad layer");
    cudaStream_t s = (cudaStream_t)stream;
    std::lock_guard<std::mutex> lk(p->mu);
    std::vector<int> es;
    for (int e = 0; e < p->n_experts; e++)
        if (p->slot_of[layer * p->n_experts + e] >= 0) es.push_back(e);
    const int n = (int)es.size();
    if (ids && n > cap) return k3c::set_error(K3C_EFULL, "pool_acquire_resident: %d resident, room for %d", n, cap);
    for (int e : es) {
        const int slot = p->slot_of[layer * p->n_experts + e];
        if (p->fill_pending[slot]) {
            if (cudaEventQuery(p->fill_ev[slot]) == cudaSuccess) {
                p->fill_pending[slot] = 0;
            } else {
                cudaError_t err = cudaStreamWaitEvent(s, p->fill_ev[slot], 0);
                if (err != cudaSuccess) return k3c::set_error(K3C_ECUDA, "pool_acquire_resident: %s", cudaGetErrorString(err));
            }
        }
    }
    cudaGetLastError();   // a not-ready event query is not an error
    for (int i = 0; i < n; i++) {
        p->pins[p->slot_of[layer * p->n_experts + es[i]]]++;
        if (ids) ids[i] = es[i];
    }
    if (dev_run_of) {
        const int b = p->stage_next;
        p->stage_next = (b + 1) % kStageRing;
        cudaEventSynchronize(p->stage_ev[b]);
        int *h = p->stage[b];
        for (int e = 0; e < p->n_experts; e++) h[e] = -1;
        for (int e : es) h[e] = p->slot_of[layer * p->n_experts + e];
        cudaError_t err = cudaMemcpyAsync(dev_run_of, h, (size_t)p->n_experts * sizeof(int), cudaMemcpyHostToDevice, s);
        if (err == cudaSuccess) err = cudaEventRecord(p->stage_ev[b], s);
        if (err != cudaSuccess) return k3c::set_error(K3C_ECUDA, "pool_acquire_resident: %s", cudaGetErrorString(err));
    }
    return n;
}

int64_t k3c_pool_trace(k3c_expert_pool *p, int32_t *out, int64_t cap) {
    if (!p) return -1;
    std::lock_guard<std::mutex> lk(p->mu);
    const int64_t n = (int64_t)p->trace.size();
    if (out)
        for (int64_t i = 0; i < n && i < cap; i++) out[i] = p->trace[(size_t)i];
    return n;
}

int k3c_pool_hist(k3c_expert_pool *p, uint32_t *out) {
    if (!p || !out) return K3C_EINVAL;
    std::lock_guard<std::mutex> lk(p->mu);
    for (size_t i = 0; i < p->hist.size(); i++) out[i] = p->hist[i];
    return K3C_OK;
}

int k3c_pool_dump_trace(k3c_expert_pool *p, const char *path) {
    if (!p || !path) return -1;
    std::lock_guard<std::mutex> lk(p->mu);
    if (p->trace.empty()) return -1;
    FILE *f = fopen(path, "wb");
    if (!f) return -1;
    const size_t n = fwrite(p->trace.data(), sizeof(int32_t), p->trace.size(), f);
    fclose(f);
    return n == p->trace.size() ? 0 : -1;
}

int k3c_pool_dump_hist(k3c_expert_pool *p, const char *path) {
    if (!p || !path) return -1;
    std::lock_guard<std::mutex> lk(p->mu);
    FILE *f = fopen(path, "w");
    if (!f) return -1;
    fprintf(f, "{\"n_layers\":%d,\"n_experts\":%d,\"counts\":{", p->n_layers, p->n_experts);
    bool first = true;
    for (int L = 0; L < p->n_layers; L++)
        for (int e = 0; e < p->n_experts; e++) {
            const uint32_t v = p->hist[(size_t)L * p->n_experts + e];
            if (!v) continue;
            fprintf(f, "%s\"%d,%d\":%u", first ? "" : ",", L, e, v);
            first = false;
        }
    fprintf(f, "}}\n");
    fclose(f);
    return 0;
}

int k3c_pool_set_pin(k3c_expert_pool *p, int layer, int expert, int pin) {
    if (!p || !key_ok(p, layer, expert)) return 0;
    std::lock_guard<std::mutex> lk(p->mu);
    const int slot = p->slot_of[layer * p->n_experts + expert];
    if (slot < 0) return 0;
    p->user_pin[slot] = pin ? 1 : 0;
    return 1;
}

void k3c_pool_reset_stats(k3c_expert_pool *p) {
    if (!p) return;
    std::lock_guard<std::mutex> lk(p->mu);
    p->st = k3c_pool_stats_t{};   // prefetch reads reset with the hits they are subtracted from
}

void k3c_pool_report(k3c_expert_pool *p, const char *label) {
    if (!p) return;
    std::lock_guard<std::mutex> lk(p->mu);
    const long long n = p->st.hits + p->st.misses;
    int resident = 0, pinned = 0;
    for (int i = 0; i < p->nslot; i++) {
        if (p->key_of[i] >= 0) resident++;
        if (p->user_pin[i] || p->pinned_forever[i]) pinned++;
    }
    printf("pool [%s]\n", label ? label : "");
    printf("  slots        : %d of %.2f MB = %.2f GB HBM (%d resident, %d pinned)\n", p->nslot,
           (double)p->stride / 1e6, (double)p->stride * p->nslot / 1e9, resident, pinned);
    printf("  requests     : %lld  hits %lld (%.2f%%)  misses %lld  evictions %lld\n", n, p->st.hits,
           n ? 100.0 * p->st.hits / n : 0.0, p->st.misses, p->st.evictions);
    if (p->st.prefetch_reads) {
        const long long served = p->st.hits > p->st.prefetch_reads ? p->st.hits - p->st.prefetch_reads : 0;
        printf("  of those hits : %lld came from the batch prefetch, i.e. copied from the host\n"
               "                  this token; TRUE resident hit rate %.2f%%\n",
               p->st.prefetch_reads, n ? 100.0 * served / n : 0.0);
    }
    printf("  copied from host: %.2f GB\n", (double)p->st.bytes_h2d / 1e9);
    fflush(stdout);
}

}  // extern "C"

// ------------------------------------------------------------------ K3ExpertSrc adapter
namespace {

struct PoolSource {
    K3ExpertSrc src;   // first member: a K3ExpertSrc* is a PoolSource*
    k3c_expert_pool *pool;
    cudaStream_t stream;
    std::vector<std::pair<int, int>> held;   // (layer, expert) pinned for the caller
    uint32_t magic;
};
constexpr uint32_t kPoolSourceMagic = 0x6b337073u;

void fill_q(const k3c_expert_pool *p, int slot, K3ExpertQ *q) {
    const k3c::PoolGeom g = k3c::pool_geom(p->hidden, p->inter);
    const unsigned char *b = p->arena + (size_t)slot * p->stride;
    q->p1 = b + g.gu_p;
    q->s1 = b + g.gu_s;
    q->p3 = nullptr;   // up is interleaved with gate inside p1 (pool format)
    q->s3 = nullptr;
    q->p2 = b + g.d_p;
    q->s2 = b + g.d_s;
}

int src_get(K3ExpertSrc *self, int layer, int expert, K3ExpertQ *out) {
    PoolSource *ps = reinterpret_cast<PoolSource *>(self);
    int slot = -1;
    if (k3c_pool_acquire(ps->pool, layer, &expert, 1, &slot, nullptr, (k3c_stream_t)ps->stream) != K3C_OK)
        return -1;
    ps->held.emplace_back(layer, expert);
    if (out) fill_q(ps->pool, slot, out);
    return 0;
}

int src_getmany(K3ExpertSrc *self, int layer, const int *ids, int n) {
    PoolSource *ps = reinterpret_cast<PoolSource *>(self);
    const int r = k3c_pool_getmany(ps->pool, layer, ids, n);
    return r < 0 ? -1 : r;
}

int src_resident(K3ExpertSrc *self, int layer, int expert, K3ExpertQ *out) {
    PoolSource *ps = reinterpret_cast<PoolSource *>(self);
    k3c_expert_pool *p = ps->pool;
    if (!key_ok(p, layer, expert)) return 0;
    std::lock_guard<std::mutex> lk(p->mu);
    const int slot = p->slot_of[layer * p->n_experts + expert];
    if (slot < 0) return 0;
    if (!out) return 1;
    if (p->fill_pending[slot]) {
        if (cudaEventQuery(p->fill_ev[slot]) == cudaSuccess) {
            p->fill_pending[slot] = 0;
        } else if (cudaStreamWaitEvent(ps->stream, p->fill_ev[slot], 0) != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        cudaGetLastError();
    }
    p->pins[slot]++;
    ps->held.emplace_back(layer, expert);
    fill_q(p, slot, out);
    return 1;
}

PoolSource *as_pool_source(const K3ExpertSrc *s) {
    if (!s || s->get != src_get) return nullptr;
    PoolSource *ps = reinterpret_cast<PoolSource *>(const_cast<K3ExpertSrc *>(s));
    return ps->magic == kPoolSourceMagic ? ps : nullptr;
}

}  // namespace

extern "C" {

K3ExpertSrc *k3c_pool_source_create(k3c_expert_pool *pool, k3c_stream_t stream) {
    k3c::clear_error();
    if (!pool) {
        k3c::set_error(K3C_EINVAL, "pool_source_create: null pool");
        return nullptr;
    }
    PoolSource *ps = new PoolSource;
    ps->src.get = src_get;
    ps->src.getmany = src_getmany;
    ps->src.resident = src_resident;
    ps->src.ctx = ps;
    ps->pool = pool;
    ps->stream = (cudaStream_t)stream;
    ps->magic = kPoolSourceMagic;
    return &ps->src;
}

int k3c_pool_source_release(K3ExpertSrc *src) {
    k3c::clear_error();
    PoolSource *ps = as_pool_source(src);
    if (!ps) return k3c::set_error(K3C_EINVAL, "pool_source_release: not a pool source");
    int rc = K3C_OK;
    for (const auto &h : ps->held) {
        const int r = k3c_pool_release(ps->pool, h.first, &h.second, 1, (k3c_stream_t)ps->stream);
        if (r != K3C_OK) rc = r;
    }
    ps->held.clear();
    return rc;
}

void k3c_pool_source_destroy(K3ExpertSrc *src) {
    PoolSource *ps = as_pool_source(src);
    if (!ps) return;
    k3c_pool_source_release(src);
    ps->magic = 0;
    delete ps;
}

k3c_stream_t k3c_pool_source_stream(const K3ExpertSrc *src) {
    PoolSource *ps = as_pool_source(src);
    return ps ? (k3c_stream_t)ps->stream : nullptr;
}

k3c_expert_pool *k3c_pool_source_pool(const K3ExpertSrc *src) {
    PoolSource *ps = as_pool_source(src);
    return ps ? ps->pool : nullptr;
}

int k3c_pool_source_slot(const K3ExpertSrc *src, const K3ExpertQ *q) {
    PoolSource *ps = as_pool_source(src);
    if (!ps || !q || !q->p1) return -1;
    const k3c_expert_pool *p = ps->pool;
    const unsigned char *a = p->arena;
    if (q->p1 < a || q->p1 >= a + (size_t)p->nslot * p->stride) return -1;
    const size_t off = (size_t)(q->p1 - a);
    return off % p->stride == 0 ? (int)(off / p->stride) : -1;
}

}  // extern "C"
