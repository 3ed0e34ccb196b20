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

#include <mutex>
#include <vector>

#include "common.cuh"

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
        if (p->pins[i] > 0) continue;
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

}  // extern "C"
