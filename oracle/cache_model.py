"""CPU model of the expert cache's bookkeeping (test infrastructure only).

Restates the reference's src/cache/k3_cache.c slot logic -- pick_victim (:46-57), admit
(:60-108), cache_getmany's reserve/publish (:131-234) and the report's hit-rate definitions
(:416-425) -- with the two adaptations the HBM pool makes, so that the pool's slot choices and
counters can be checked exactly:
  * a batch prefetch publishes each expert when its copy is issued (the copy's completion is
    tracked by an event, not by the caller waiting), in request order (host memory has no
    disk offsets to sort by), with one clock tick per slot;
  * get() pins the slot until release() (the reference keeps the current token's experts by
    requiring nslot >= topk + 1; the pool pins them explicitly).
"""

EMPTY, INFLIGHT = -1, -2


class CacheModel:
    def __init__(self, n_layers, n_experts, nslot):
        self.n_experts = n_experts
        self.slot_of = {}
        self.key_of = [EMPTY] * nslot
        self.pins = [0] * nslot
        self.used_at = [0] * nslot
        self.clock = 0
        self.hits = self.misses = self.evictions = self.prefetch_reads = 0

    def _victim(self):  # k3_cache.c:46-57
        best, oldest = -1, None
        for i, k in enumerate(self.key_of):
            if k == INFLIGHT:
                continue
            if k == EMPTY:
                return i
            if self.pins[i] > 0:
                continue
            if oldest is None or self.used_at[i] < oldest:
                oldest, best = self.used_at[i], i
        return best

    def _fill(self, key):
        s = self._victim()
        if s < 0:
            raise RuntimeError("every slot is pinned")
        if self.key_of[s] >= 0:
            del self.slot_of[self.key_of[s]]
            self.evictions += 1
        self.key_of[s] = key
        self.slot_of[key] = s
        self.clock += 1
        self.used_at[s] = self.clock
        return s

    def getmany(self, layer, ids):  # k3_cache.c:131-234 (request order, publish on issue)
        n = 0
        for e in ids:
            key = layer * self.n_experts + e
            if key in self.slot_of:
                continue
            self._fill(key)
            self.prefetch_reads += 1
            n += 1
        return n

    def acquire(self, layer, ids):  # admit, k3_cache.c:60-108, per request, plus a pin
        out = []
        for e in ids:
            key = layer * self.n_experts + e
            s = self.slot_of.get(key, -1)
            if s >= 0:
                self.hits += 1
                self.clock += 1
                self.used_at[s] = self.clock
            else:
                self.misses += 1
                s = self._fill(key)
            self.pins[s] += 1
            out.append(s)
        return out

    def release(self, layer, ids):
        for e in ids:
            s = self.slot_of.get(layer * self.n_experts + e, -1)
            if s >= 0 and self.pins[s] > 0:
                self.pins[s] -= 1

    def stats(self):
        n = self.hits + self.misses
        return {"hits": self.hits, "misses": self.misses, "evictions": self.evictions,
                "prefetch_reads": self.prefetch_reads,
                "hit_rate": self.hits / n if n else None,
                "true_hit_rate": max(self.hits - self.prefetch_reads, 0) / n if n else None}
