// moe_pool.cu -- MoE decode on the 5th-generation tensor cores (tcgen05, kind::mxf8f6f4).
//
// The routed experts stay in MXFP4: TMA streams the packed E2M1 nibbles straight into
// shared memory (the 16U4_ALIGN16B tensor-map type places each 8-byte group of 16 nibbles
// in a 16-byte slot, the layout the f8f6f4 MMA reads), the E8M0 scales go to TMEM through
// tcgen05.cp, and one elected thread issues tcgen05.mma with the weights as the M=128
// operand and the tokens as N. No instruction decodes a nibble.
//
// Activations enter the MMA as J terms of E4M3 with one UE8M0 scale per 32 elements:
// term 1 rounds x to E4M3 under a power-of-two block scale, each further term rounds what
// the previous terms left over, so J terms carry about 4J significant bits relative to the
// block maximum. bf16 inputs need J=2-3; J is the precision knob of the path.
//
// Pool format of one expert run (hidden H, inter I; same byte count as the reference's
// run, 23,396,352 B at 7168/2048):
//   GU packed  [2I rows][H/2]    row block b of 128 = gate rows 64b..64b+63, then up rows
//                                64b..64b+63, so one M=128 tile holds matching gate/up rows
//   GU scales  [2I/128][H/128] atoms of 512 B
//   D  packed  [H rows][I/2]
//   D  scales  [H/128][I/128] atoms of 512 B
// A scale atom covers 128 rows x 4 groups of 32: byte 16*(m%32) + 4*(m/32) + g, the layout
// the 32x128b.warpx4 TMEM copy expects. Groups whose scale byte is 255 (the reference zeroes
// them, src/core/k3_ops.c:1519) are stored as zero nibbles with scale 127.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdlib.h>

#include "common.cuh"
#include "tc_common.cuh"
#include "tc_host.cuh"
#include "pool_common.cuh"

namespace k3c {

int launch_router(int *idx, float *w, float *scores, const void *x, int x_dtype, const void *W, int w_dtype,
                  const float *bias, int hidden, int n_experts, int topk, int renorm, float routed_scale,
                  int ntok, double *part, cudaStream_t s);
size_t router_scratch_bytes(int hidden, int n_experts, int ntok);
int launch_moe_combine(float *out, const float *contrib, const float *wt, const uint8_t *dropped,
                       int ntok, int topk, int hidden, int has_shared, cudaStream_t s);

// ------------------------------------------------------------------ repack
// Reference layout (K3ExpertQ, device addresses) -> one pool-format run.
__global__ void k_pool_pack(uint8_t *__restrict__ run, K3ExpertQ src, int H, int I) {
    const PoolGeom g = pool_geom(H, I);
    const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
    const size_t nthr = (size_t)gridDim.x * blockDim.x;
    const int hg = H / 32, ig = I / 32;
    // GU packed: 16-byte chunks (one scale group each)
    for (size_t c = tid; c < (size_t)2 * I * hg; c += nthr) {
        const int R = (int)(c / hg), grp = (int)(c % hg);
        int which, row;
        gu_source(R, which, row);
        const uint8_t *sp = which ? src.p3 : src.p1;
        const uint8_t *ss = which ? src.s3 : src.s1;
        uint4 v = *reinterpret_cast<const uint4 *>(sp + (size_t)row * (H / 2) + (size_t)grp * 16);
        if (ss[(size_t)row * hg + grp] == 255) v = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4 *>(run + g.gu_p + (size_t)R * (H / 2) + (size_t)grp * 16) = v;
    }
    // D packed
    for (size_t c = tid; c < (size_t)H * ig; c += nthr) {
        const int h = (int)(c / ig), grp = (int)(c % ig);
        uint4 v = *reinterpret_cast<const uint4 *>(src.p2 + (size_t)h * (I / 2) + (size_t)grp * 16);
        if (src.s2[(size_t)h * ig + grp] == 255) v = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4 *>(run + g.d_p + (size_t)h * (I / 2) + (size_t)grp * 16) = v;
    }
    // GU scale atoms
    for (size_t b = tid; b < (size_t)2 * I * hg; b += nthr) {
        const int R = (int)(b / hg), grp = (int)(b % hg);
        int which, row;
        gu_source(R, which, row);
        uint8_t s = (which ? src.s3 : src.s1)[(size_t)row * hg + grp];
        if (s == 255) s = 127;
        const size_t atom = (size_t)(R / 128) * (H / 128) + grp / 4;
        run[g.gu_s + atom * 512 + atom_byte(R % 128, grp % 4)] = s;
    }
    // D scale atoms
    for (size_t b = tid; b < (size_t)H * ig; b += nthr) {
        const int h = (int)(b / ig), grp = (int)(b % ig);
        uint8_t s = src.s2[(size_t)h * ig + grp];
        if (s == 255) s = 127;
        const size_t atom = (size_t)(h / 128) * (I / 128) + grp / 4;
        run[g.d_s + atom * 512 + atom_byte(h % 128, grp % 4)] = s;
    }
}

// ------------------------------------------------------------------ activation terms
// x [ntok][H] -> x_q [J*NT][H] E4M3, row j*NT + t holding term j of token t, and the scale
// atoms x_sf [H/128][512] over those rows (J*NT <= 96 rows: one atom row).
template <int J, typename XT>
__global__ void __launch_bounds__(256) k_quant_x(uint8_t *__restrict__ xq, uint8_t *__restrict__ xsf,
                                                 const XT *__restrict__ x, int ntok, int H, int NT) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int blk = blockIdx.x * 8 + warp;  // 32-element block index
    const int t = blockIdx.y;
    if (blk * 32 >= H || t >= ntok) return;
    const int k = blk * 32 + lane;
    float a;
    if constexpr (sizeof(XT) == 2) a = bf16_bits_to_f32(x[(size_t)t * H + k]);
    else a = x[(size_t)t * H + k];
    quantize_block<J>(
        a, [&](int j, uint32_t q) { xq[((size_t)j * NT + t) * H + k] = (uint8_t)q; },
        [&](int j, uint32_t sf) {
            xsf[(size_t)(blk / 4) * 512 + atom_byte(j * NT + t, blk % 4)] = (uint8_t)sf;
        });
}

// ------------------------------------------------------------------ plan (tc)
struct SlotTc {
    int run, ntok;
};

// Same grouping as the CUDA-core plan, slot-major with 32 pair rows per slot: one slot per
// selected resident expert in expert order, then the shared expert. One block; every step
// is parallel over pairs or experts (slot numbers by a block-wide prefix count), and a pair's
// row within its slot is its rank among the earlier pairs of the same expert.
__global__ void __launch_bounds__(1024) k_moe_plan_tc(int *__restrict__ n_slots, SlotTc *__restrict__ slots,
                                                      int *__restrict__ pair_tok, int *__restrict__ pair_k,
                                                      uint8_t *__restrict__ dropped, const int *__restrict__ idx,
                                                      int ntok, int topk, const int *__restrict__ run_of,
                                                      int n_experts, int n_runs, int shared_run,
                                                      int *__restrict__ drops) {
    extern __shared__ int sm[];
    int *cnt = sm, *slot_of = sm + n_experts;        // [E], [E]
    int *pe = slot_of + n_experts;                   // [P] expert of each kept pair, -1 if dropped
    __shared__ int warp_sum[32];
    const int P = ntok * topk;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int e = threadIdx.x; e < n_experts; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < P; i += blockDim.x) {
        const int e = idx[i];
        // a run index outside the arena is treated as not resident: the kernels form raw
        // scale addresses from it
        const bool ok = e >= 0 && e < n_experts && run_of[e] >= 0 && run_of[e] < n_runs;
        dropped[i] = ok ? 0 : 1;
        pe[i] = ok ? e : -1;
        if (ok) atomicAdd(&cnt[e], 1);
        else if (drops) atomicAdd(drops, 1);
    }
    __syncthreads();
    // slot numbers: exclusive prefix count of used experts, in chunks of blockDim experts
    int base = 0;
    for (int e0 = 0; e0 < n_experts; e0 += blockDim.x) {
        const int e = e0 + threadIdx.x;
        const bool used = e < n_experts && cnt[e] > 0;
        const unsigned m = __ballot_sync(0xffffffffu, used);
        if (lane == 0) warp_sum[warp] = __popc(m);
        __syncthreads();
        int before = base;
        for (int w = 0; w < warp; w++) before += warp_sum[w];
        int total = 0;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) total += warp_sum[w];
        if (e < n_experts) {
            const int sl = before + __popc(m & ((1u << lane) - 1u));
            slot_of[e] = used ? sl : -1;
            if (used) {
                slots[sl].run = run_of[e];
                slots[sl].ntok = cnt[e];
            }
        }
        base += total;
        __syncthreads();   // warp_sum is rewritten by the next chunk
    }
    if (shared_run >= 0) {
        for (int t = threadIdx.x; t < ntok; t += blockDim.x) {
            pair_tok[base * 32 + t] = t;
            pair_k[base * 32 + t] = topk;
        }
        if (threadIdx.x == 0) {
            slots[base].run = shared_run;
            slots[base].ntok = ntok;
        }
    }
    if (threadIdx.x == 0) *n_slots = base + (shared_run >= 0 ? 1 : 0);
    for (int i = threadIdx.x; i < P; i += blockDim.x) {
        const int e = pe[i];
        if (e < 0) continue;
        int rank = 0;
        for (int k = 0; k < i; k++) rank += pe[k] == e;
        const int pos = slot_of[e] * 32 + rank;
        pair_tok[pos] = i / topk;
        pair_k[pos] = i % topk;
    }
}

// ------------------------------------------------------------------ persistent tcgen05 kernel
// Persistent CTAs (two per SM) loop over work items (slot, row tile). Six warps:
//   warp 0      TMA producer: one thread streams A (weights), B (the activation terms) and
//               their scale atoms through a STAGES-deep ring, continuously across items;
//   warp 1      MMA issuer: one thread copies the two scale atoms of a K tile into TMEM and
//               issues one tcgen05 MMA per 32-element K block into one of two accumulators;
//   warps 2-5   epilogue: wait for an accumulator, read it with tcgen05.ld (warp w owns TMEM
//               lanes 32*(w%4)..+31), hand it back, then run the item's epilogue while the
//               MMA warp fills the other accumulator.
// The J activation terms of each token are stacked as J*NT rows of the B operand (row
// j*NT + t = term j of token t), each row with its own block scales, so one MMA with
// N = J*NT covers all terms and the epilogue adds the J partial columns of a token.
// GU items: 64 gate + 64 up rows for output columns [64*rt, 64*rt+64); the epilogue applies
// the activation and requantises it into the D stage's operand. D items: 128 down rows x
// the slot's pairs; the epilogue writes each pair's unweighted expert output to contrib.
// GU hands items out round robin (they are all the same size). D runs as a programmatic
// dependent of GU and starts on the SMs that GU's CTAs leave: its producer takes items from
// a queue shared by all CTAs (slot-major, so the slots GU finished first come first), passes
// them to the MMA and epilogue warps through a small ring in shared memory, and waits only
// for the GU row tiles of the item's own slot (a per-slot counter GU releases), so the down
// projections fill the SMs while the last GU items finish.
constexpr int TC_A_BYTES = 128 * 128;   // shared-memory footprint of a padded E2M1 tile
constexpr int TC_A_TX = 128 * 128 / 2;  // its TMA transaction bytes: 4 bits per element
constexpr int TC_THREADS = 192;
constexpr int TC_IRING = 4;             // D: items in flight between the producer and the consumers

__host__ __device__ constexpr uint32_t pow2_cols(uint32_t n) {
    return n <= 32 ? 32 : n <= 64 ? 64 : n <= 128 ? 128 : n <= 256 ? 256 : 512;
}

template <int J, int NT, int STAGES>
struct TcCfg {
    static constexpr int NCOL = J * NT;                   // MMA N
    static constexpr int B_BYTES = NCOL * 128;
    static constexpr int STAGE = TC_A_BYTES + B_BYTES + 1024;   // + SFA and SFB atoms
    static constexpr int TILE = 128 * (NT + 1) * 4;       // epilogue staging [128][NT+1] fp32
    static constexpr int BYTES = STAGES * STAGE + TILE + 256 + 1024;
    // mbarriers (full/empty per stage, two accumulator pairs, the item ring's pair), the TMEM
    // address and the item ring share the 256 bytes after the staging tile
    static_assert(8 * (2 * STAGES + 4 + 2 * TC_IRING) + 4 + 4 * TC_IRING <= 256, "barrier area");
    static constexpr uint32_t SF_COL = 2 * NCOL;          // after the two accumulators
    static constexpr uint32_t TMEM_COLS = pow2_cols(2 * NCOL + 16);
    static constexpr uint32_t TX = TC_A_TX + B_BYTES + 1024;
};

struct TcArgs {
    const int *n_slots;
    const SlotTc *slots;
    const int *pair_tok, *pair_k;
    const uint8_t *arena;
    size_t run_stride;
    const uint8_t *x_sf;     // GU B scale atoms [H/128][512] (row j*NT + t)
    uint8_t *act_q;          // GU output / D operand: [S][J*NT][I]
    uint8_t *act_sf;         // [S][I/128][512], row j*NT + pair
    float *contrib;          // D output [T][topk+1][H]
    int kstride;             // topk + 1
    int H, I, act;
    int *err;
    int *d_next;             // D: next item of the queue (zero at launch)
    int *gu_done;            // [S] GU row tiles of each slot written (zero at launch)
};

using tc::l2_evict_first_policy;
using tc::named_bar_sync;
using tc::tc_check;
using tc::tma_load_3d_hint;
using tc::tmem_ld16;

template <int J, int NT, int STAGES, bool GU>
__global__ void __launch_bounds__(TC_THREADS) k_tc_moe(const __grid_constant__ CUtensorMap tmW,
                                                      const __grid_constant__ CUtensorMap tmB,
                                                      TcArgs p) {
    using Cfg = TcCfg<J, NT, STAGES>;
    constexpr int NCOL = Cfg::NCOL;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    float *tile = reinterpret_cast<float *>(smem + STAGES * Cfg::STAGE);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGES * Cfg::STAGE + Cfg::TILE);
    uint64_t *full = bars, *empty = bars + STAGES, *tfull = bars + 2 * STAGES, *tempty = tfull + 2;
    uint64_t *ifull = tempty + 2, *iempty = ifull + TC_IRING;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(iempty + TC_IRING);
    int *iring = reinterpret_cast<int *>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if constexpr (GU) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");   // D may be scheduled
    if (threadIdx.x == 0) {
        for (int i = 0; i < 2 * STAGES; i++) tc::mbar_init(&bars[i], 1);
        tc::mbar_init(&tfull[0], 1);
        tc::mbar_init(&tfull[1], 1);
        tc::mbar_init(&tempty[0], 4);
        tc::mbar_init(&tempty[1], 4);
        for (int i = 0; i < TC_IRING; i++) {
            tc::mbar_init(&ifull[i], 1);
            tc::mbar_init(&iempty[i], 5);   // the MMA thread and one lane of each epilogue warp
        }
        tc::fence_mbar_init();
    }
    if (warp == 1) tc::tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int n_slots = *p.n_slots;
    const int RT = GU ? (2 * p.I) / 128 : p.H / 128;   // row tiles per slot
    const int KT = GU ? p.H / 128 : p.I / 128;         // K tiles per item
    const int n_items = n_slots * RT;
    const PoolGeom g = pool_geom(p.H, p.I);
    const size_t sf_off = GU ? g.gu_s : g.d_s;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------------ producer
        bool ok = tc_check((tc::smem_u32(smem) & 1023) == 0, p.err, 10);
        tc::prefetch_tmap(&tmW);
        tc::prefetch_tmap(&tmB);
        const uint64_t pol = l2_evict_first_policy();
        uint32_t kiter = 0;
        int ready_s = -1;   // D: the last slot whose activation terms were seen complete
        for (uint32_t li = 0; ok; li++) {
            int it;
            if constexpr (GU) {
                it = (int)(blockIdx.x + li * gridDim.x);
                if (it >= n_items) break;
            } else {
                // take the next item of the queue and hand it to the MMA and epilogue warps
                const uint32_t r = li % TC_IRING;
                if (li >= TC_IRING && !tc::mbar_wait(&iempty[r], (li / TC_IRING - 1) & 1u, p.err, 11)) {
                    ok = false;
                    break;
                }
                it = atomicAdd(p.d_next, 1);
                iring[r] = it < n_items ? it : -1;
                tc::mbar_arrive(&ifull[r]);
                if (it >= n_items) break;
            }
            const int s = it / RT, rt = it % RT;
            const SlotTc sl = p.slots[s];
            const uint8_t *sfa = p.arena + (size_t)sl.run * p.run_stride + sf_off + (size_t)rt * KT * 512;
            const uint8_t *sfb = GU ? p.x_sf : p.act_sf + (size_t)s * KT * 512;
            const int b_row = GU ? 0 : NCOL * s;
            if constexpr (!GU) {
                // the slot's activation terms are complete once all of its GU row tiles are
                if (s != ready_s) {
                    if (!tc::wait_count(p.gu_done + s, (2 * p.I) / 128, p.err, 12)) {
                        ok = false;
                        break;
                    }
                    tc::fence_proxy_async_global();
                    ready_s = s;
                }
            }
            for (int kt = 0; kt < KT; kt++, kiter++) {
                const int st = kiter % STAGES;
                const uint32_t ph = (kiter / STAGES) & 1u;
                if (kiter >= STAGES && !tc::mbar_wait(&empty[st], ph ^ 1u, p.err, 1)) { ok = false; break; }
                uint8_t *sa = smem + st * Cfg::STAGE;
                uint8_t *sb = sa + TC_A_BYTES;
                uint8_t *ssf = sb + Cfg::B_BYTES;
                tc::mbar_expect_tx(&full[st], Cfg::TX);
                tma_load_3d_hint(sa, &tmW, &full[st], kt * 128, rt * 128, sl.run, pol);
                tc::tma_load_3d(sb, &tmB, &full[st], kt * 128, b_row, 0);
                tc::bulk_load(ssf, sfa + (size_t)kt * 512, 512, &full[st]);
                tc::bulk_load(ssf + 512, sfb + (size_t)kt * 512, 512, &full[st]);
            }
        }
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------------------ MMA issuer
        uint32_t kiter = 0;
        bool ok = true;
        const uint32_t idesc0 = tc::idesc_mxf8f6f4(tc::FMT_E2M1, tc::FMT_E4M3, NCOL, 0, 0);
        for (uint32_t li = 0; ok; li++) {
            if constexpr (GU) {
                if ((int)(blockIdx.x + li * gridDim.x) >= n_items) break;
            } else {
                const uint32_t r = li % TC_IRING;
                if (!tc::mbar_wait(&ifull[r], (li / TC_IRING) & 1u, p.err, 13)) break;
                const int it = iring[r];
                tc::mbar_arrive(&iempty[r]);
                if (it < 0) break;
            }
            const uint32_t a = li & 1u, use = li >> 1;
            if (use >= 1 && !tc::mbar_wait(&tempty[a], (use - 1) & 1u, p.err, 4)) { ok = false; break; }
            tc::tc_fence_after();
            const uint32_t d = tmem + a * NCOL;
            for (int kt = 0; kt < KT; kt++, kiter++) {
                const int st = kiter % STAGES;
                const uint32_t ph = (kiter / STAGES) & 1u;
                if (!tc::mbar_wait(&full[st], ph, p.err, 2)) { ok = false; break; }
                tc::tc_fence_after();
                uint8_t *sa = smem + st * Cfg::STAGE;
                uint8_t *sb = sa + TC_A_BYTES;
                uint8_t *ssf = sb + Cfg::B_BYTES;
                const uint32_t sfc = tmem + Cfg::SF_COL + 8u * (kiter & 1u);
                tc::tc_cp_sf(sfc, tc::desc_sf_atom(tc::smem_u32(ssf)));
                tc::tc_cp_sf(sfc + 4, tc::desc_sf_atom(tc::smem_u32(ssf + 512)));
#pragma unroll
                for (int kb = 0; kb < 4; kb++) {
                    const uint64_t da = tc::desc_kmajor_sw128(tc::smem_u32(sa) + 32 * kb);
                    const uint64_t db = tc::desc_kmajor_sw128(tc::smem_u32(sb) + 32 * kb);
                    const uint32_t id = idesc0 | ((uint32_t)kb << 4) | ((uint32_t)kb << 29);
                    tc::tc_mma_mx(d, da, db, id, sfc | ((uint32_t)kb << 30), (sfc + 4) | ((uint32_t)kb << 30),
                                  (kt | kb) != 0);
                }
                tc::tc_commit(&empty[st]);
            }
            if (ok) tc::tc_commit(&tfull[a]);
        }
    } else if (warp >= 2) {
        // ------------------------------------------------------------ epilogue
        // GU: every epilogue warp runs every item and every named barrier even after a failed
        // wait (it then skips the TMEM read and the work), so the barriers cannot strand a
        // warp; once an error is recorded the remaining waits return at once. D has no named
        // barriers: a warp leaves the queue at the first failed wait.
        const int q = warp & 3;                 // TMEM lane quadrant
        const int row = 32 * q + lane;          // row within the 128-row tile
        for (uint32_t li = 0;; li++) {
            int it;
            if constexpr (GU) {
                it = (int)(blockIdx.x + li * gridDim.x);
                if (it >= n_items) break;
            } else {
                const uint32_t r = li % TC_IRING;
                if (*(volatile int *)p.err != 0 || !tc::mbar_wait(&ifull[r], (li / TC_IRING) & 1u, p.err, 14)) break;
                it = iring[r];
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&iempty[r]);
                if (it < 0) break;
            }
            const int s = it / RT, rt = it % RT;
            const uint32_t a = li & 1u;
            const bool ok = *(volatile int *)p.err == 0 && tc::mbar_wait(&tfull[a], (li >> 1) & 1u, p.err, 3);
            float val[NT];
            if (ok) {
                tc::tc_fence_after();
                uint32_t v[NCOL];
#pragma unroll
                for (int c = 0; c < NCOL; c += 16)
                    tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + a * NCOL + c, v + c);
                tc::tmem_ld_wait();
                tc::tc_fence_before();
                if (lane == 0) tc::mbar_arrive(&tempty[a]);
#pragma unroll
                for (int c = 0; c < NT; c++) {
                    float acc = __uint_as_float(v[c]);
#pragma unroll
                    for (int j = 1; j < J; j++) acc += __uint_as_float(v[j * NT + c]);
                    val[c] = acc;
                }
            }
            const SlotTc sl = p.slots[s];
            if constexpr (GU) {
                if (ok) {
#pragma unroll
                    for (int c = 0; c < NT; c++) tile[row * (NT + 1) + c] = val[c];
                }
                named_bar_sync(1, 128);
                if (ok && q < 2) {               // gate rows 0..63 (warps 4 and 5)
                    const int col = 64 * rt + row;   // output column in [0, I)
                    const int KTd = p.I / 128;
                    for (int pl = 0; pl < sl.ntok; pl++) {
                        const int tok = p.pair_tok[s * 32 + pl];
                        const float av = act_apply(tile[row * (NT + 1) + tok], tile[(row + 64) * (NT + 1) + tok], p.act);
                        quantize_block<J>(
                            av,
                            [&](int j, uint32_t qv) {
                                p.act_q[((size_t)s * NCOL + j * NT + pl) * p.I + col] = (uint8_t)qv;
                            },
                            [&](int j, uint32_t sf) {
                                p.act_sf[((size_t)s * KTd + col / 128) * 512 + atom_byte(j * NT + pl, (col % 128) / 32)] =
                                    (uint8_t)sf;
                            });
                    }
                    // the down kernel reads these bytes with TMA in other CTAs
                    tc::fence_proxy_async_global();
                    __threadfence();
                }
                named_bar_sync(1, 128);          // the tile is reused by the next item
                // this row tile of slot s is written (also after a failed wait: the error code
                // is set, and the down kernel should not wait out its timeout as well)
                if (q == 2 && lane == 0) tc::red_release_add1(p.gu_done + s);
            } else if (ok) {
                const int h = 128 * rt + row;
#pragma unroll
                for (int pl = 0; pl < NT; pl++) {
                    if (pl < sl.ntok) {
                        const int prow = s * 32 + pl;
                        p.contrib[((size_t)p.pair_tok[prow] * p.kstride + p.pair_k[prow]) * p.H + h] = val[pl];
                    }
                }
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) tc::tmem_dealloc(tmem, Cfg::TMEM_COLS);
}

// ------------------------------------------------------------------ host side
struct TcBufs {
    int *n_slots;
    SlotTc *slots;
    int *pair_tok, *pair_k;
    uint8_t *dropped;
    float *wt, *contrib;
    int *idx;
    uint8_t *xq, *xsf, *actq, *actsf;
    int *err;
    int max_slots;
};

static bool carve_tc(Carve &cv, TcBufs &b, const k3c_moe_pool_layer *L, int ntok) {
    const int P = ntok * L->topk;
    const int H = L->hidden, I = L->inter, J = L->terms;
    b.max_slots = (P < L->n_experts ? P : L->n_experts) + 1;
    b.n_slots = cv.take<int>(1);
    // error code, the down kernel's queue head, then the per-slot GU counters: zeroed together
    b.err = cv.take<int>(2 + (size_t)b.max_slots);
    b.slots = cv.take<SlotTc>(b.max_slots);
    b.pair_tok = cv.take<int>((size_t)b.max_slots * 32);
    b.pair_k = cv.take<int>((size_t)b.max_slots * 32);
    b.dropped = cv.take<uint8_t>(P);
    b.idx = cv.take<int>(P);
    b.wt = cv.take<float>(P);
    // contrib is first written by the down kernel, after routing: the router's logit chunks
    // share its space
    const size_t nc = (size_t)ntok * (L->topk + 1) * H;
    const size_t np = router_scratch_bytes(H, L->n_experts, ntok) / sizeof(float);
    b.contrib = cv.take<float>(nc > np ? nc : np);
    b.xq = cv.take<uint8_t>((size_t)J * 32 * H, 1024);
    b.xsf = cv.take<uint8_t>((size_t)(H / 128) * 512, 1024);
    b.actq = cv.take<uint8_t>((size_t)b.max_slots * J * 32 * I, 1024);
    b.actsf = cv.take<uint8_t>((size_t)b.max_slots * (I / 128) * 512, 1024);
    return b.n_slots && b.err && b.slots && b.pair_tok && b.pair_k && b.dropped &&
           b.idx && b.wt && b.contrib && b.xq && b.xsf && b.actq && b.actsf;
}

static char *const kSizing = reinterpret_cast<char *>(4096);

size_t moe_decode_tc_scratch(const k3c_moe_pool_layer *L, int ntok) {
    Carve cv{kSizing, (size_t)-1 / 2, 0};
    TcBufs b;
    carve_tc(cv, b, L, ntok);
    return cv.used + 1024;
}

template <int J, int NT, int STAGES>
static int launch_tc_stages(const TcBufs &b, const k3c_moe_pool_layer *L, cudaStream_t s) {
    using Cfg = TcCfg<J, NT, STAGES>;
    static_assert(2 * Cfg::BYTES <= 228 * 1024, "two CTAs per SM");
    const int H = L->hidden, I = L->inter;
    const PoolGeom g = pool_geom(H, I);
    CUtensorMap tmGU, tmD, tmX, tmAct;
    K3C_TRY(make_map3(&tmGU, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, L->arena + g.gu_p, H, 2 * I, L->n_runs,
                      H / 2, L->run_stride, 128, 128));
    K3C_TRY(make_map3(&tmD, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, L->arena + g.d_p, I, H, L->n_runs, I / 2,
                      L->run_stride, 128, 128));
    constexpr int NCOL = Cfg::NCOL;
    K3C_TRY(make_map3(&tmX, CU_TENSOR_MAP_DATA_TYPE_UINT8, b.xq, H, NCOL, 1, H, (uint64_t)NCOL * H, 128, NCOL));
    K3C_TRY(make_map3(&tmAct, CU_TENSOR_MAP_DATA_TYPE_UINT8, b.actq, I, (uint64_t)b.max_slots * NCOL, 1, I,
                      (uint64_t)b.max_slots * NCOL * I, 128, NCOL));
    TcArgs a;
    a.n_slots = b.n_slots;
    a.slots = b.slots;
    a.pair_tok = b.pair_tok;
    a.pair_k = b.pair_k;
    a.arena = L->arena;
    a.run_stride = L->run_stride;
    a.x_sf = b.xsf;
    a.act_q = b.actq;
    a.act_sf = b.actsf;
    a.contrib = b.contrib;
    a.kstride = L->topk + 1;
    a.H = H;
    a.I = I;
    a.act = L->act;
    a.err = b.err;
    a.d_next = b.err + 1;
    a.gu_done = b.err + 2;
    auto kgu = k_tc_moe<J, NT, STAGES, true>;
    auto kd = k_tc_moe<J, NT, STAGES, false>;
    K3C_TRY_CUDA(cudaFuncSetAttribute(kgu, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::BYTES));
    K3C_TRY_CUDA(cudaFuncSetAttribute(kd, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::BYTES));
    // all of the unified L1/shared storage as shared memory, so two CTAs fit per SM
    K3C_TRY_CUDA(cudaFuncSetAttribute(kgu, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    K3C_TRY_CUDA(cudaFuncSetAttribute(kd, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    // CTAs per SM from the shared-memory budget (228 KB per SM, 1 KB reserved per CTA); the
    // CTAs are independent, so a CTA that does not fit simply starts when another ends.
    const int per_sm = (228 * 1024) / (Cfg::BYTES + 1024) >= 2 ? 2 : 1;
    const int grid = sm_count() * per_sm;
    stage_begin(STAGE_EXPERTS, s);
    kgu<<<grid, TC_THREADS, Cfg::BYTES, s>>>(tmGU, tmX, a);
    K3C_CHECK_LAUNCH();
    K3C_TRY_CUDA(launch_pdl(kd, dim3(grid), dim3(TC_THREADS), Cfg::BYTES, s, tmD, tmAct, a));
    K3C_CHECK_LAUNCH();
    stage_end(STAGE_EXPERTS, s);
    return K3C_OK;
}

template <int J>
static int launch_quant_x(const TcBufs &b, const void *x, int x_dtype, int ntok, int H, int NT, cudaStream_t s) {
    dim3 gq(H / 256 + (H % 256 ? 1 : 0), ntok);
    if (x_dtype == K3C_BF16) k_quant_x<J, uint16_t><<<gq, 256, 0, s>>>(b.xq, b.xsf, (const uint16_t *)x, ntok, H, NT);
    else if (x_dtype == K3C_F32) k_quant_x<J, float><<<gq, 256, 0, s>>>(b.xq, b.xsf, (const float *)x, ntok, H, NT);
    else return set_error(K3C_EINVAL, "moe_decode_tc: x_dtype=%d", x_dtype);
    K3C_CHECK_LAUNCH();
    return K3C_OK;
}

// routed: idx_out/wt_out hold the routing on entry and the router is skipped.
int launch_moe_decode_tc(float *out, const void *x, int x_dtype, int ntok, const k3c_moe_pool_layer *L,
                         int *idx_out, float *wt_out, int *drops, void *scratch, size_t scratch_bytes,
                         cudaStream_t s, bool routed = false) {
    if (!L) return set_error(K3C_EINVAL, "moe_decode_tc: null layer");
    const int H = L->hidden, I = L->inter;
    if (H <= 0 || I <= 0 || H % 128 || I % 128)
        return set_error(K3C_EINVAL, "moe_decode_tc: hidden=%d inter=%d must be multiples of 128", H, I);
    if (L->terms < 1 || L->terms > 3) return set_error(K3C_EINVAL, "moe_decode_tc: terms=%d outside 1..3", L->terms);
    if (ntok <= 0) return K3C_OK;
    if (ntok > 32) return set_error(K3C_EINVAL, "moe_decode_tc: ntok=%d > 32", ntok);
    if (L->topk <= 0 || L->topk > K3_MAX_TOPK || L->topk > L->n_experts)
        return set_error(K3C_EINVAL, "moe_decode_tc: topk=%d", L->topk);
    if (!L->arena || !L->run_of || L->n_runs <= 0 || L->run_stride % 256 ||
        L->run_stride < pool_geom(H, I).run || ((uintptr_t)L->arena & 255) || L->shared_run >= L->n_runs)
        return set_error(K3C_EINVAL, "moe_decode_tc: bad arena");
    Carve cv{(char *)scratch, scratch_bytes, 0};
    TcBufs b;
    if (!carve_tc(cv, b, L, ntok)) return set_error(K3C_EINVAL, "moe_decode_tc: scratch too small (%zu)", scratch_bytes);
    int *idx = idx_out ? idx_out : b.idx;
    float *wt = wt_out ? wt_out : b.wt;
    if (routed && (!idx_out || !wt_out)) return set_error(K3C_EINVAL, "moe_decode_tc_routed: null routing");
    K3C_TRY_CUDA(cudaMemsetAsync(b.err, 0, (2 + (size_t)b.max_slots) * sizeof(int), s));
    if (!routed) {
        stage_begin(STAGE_ROUTER, s);
        K3C_TRY(launch_router(idx, wt, nullptr, x, x_dtype, L->router_w, L->router_dtype, L->router_bias, H,
                              L->n_experts, L->topk, L->renorm, L->routed_scale, ntok,
                              reinterpret_cast<double *>(b.contrib), s));
        stage_end(STAGE_ROUTER, s);
    }
    const size_t psmem = ((size_t)L->n_experts * 2 + (size_t)ntok * L->topk) * sizeof(int);
    if (psmem > 48 * 1024)
        K3C_TRY_CUDA(cudaFuncSetAttribute(k_moe_plan_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)psmem));
    k_moe_plan_tc<<<1, 1024, psmem, s>>>(b.n_slots, b.slots, b.pair_tok, b.pair_k, b.dropped, idx, ntok,
                                         L->topk, L->run_of, L->n_experts, L->n_runs, L->shared_run, drops);
    K3C_CHECK_LAUNCH();
    const bool n16 = ntok <= 16;
    const int NT = n16 ? 16 : 32;
    switch (L->terms) {
    case 1:
        K3C_TRY(launch_quant_x<1>(b, x, x_dtype, ntok, H, NT, s));
        K3C_TRY(n16 ? (launch_tc_stages<1, 16, 5>(b, L, s)) : (launch_tc_stages<1, 32, 4>(b, L, s)));
        break;
    case 2:
        K3C_TRY(launch_quant_x<2>(b, x, x_dtype, ntok, H, NT, s));
        K3C_TRY(n16 ? (launch_tc_stages<2, 16, 4>(b, L, s)) : (launch_tc_stages<2, 32, 3>(b, L, s)));
        break;
    default:
        K3C_TRY(launch_quant_x<3>(b, x, x_dtype, ntok, H, NT, s));
        K3C_TRY(n16 ? (launch_tc_stages<3, 16, 4>(b, L, s)) : (launch_tc_stages<3, 32, 3>(b, L, s)));
        break;
    }
    K3C_TRY(launch_moe_combine(out, b.contrib, wt, b.dropped, ntok, L->topk, H, L->shared_run >= 0 ? 1 : 0, s));
    // K3C_SYNC_CHECK=1: synchronise and report the kernels' own error code (a bounded wait
    // that gave up, or a failed alignment self-check). Off by default: it costs a host sync.
    static const int sync_check = getenv("K3C_SYNC_CHECK") ? 1 : 0;
    if (sync_check) {
        int code = 0;
        K3C_TRY_CUDA(cudaMemcpyAsync(&code, b.err, sizeof(int), cudaMemcpyDeviceToHost, s));
        K3C_TRY_CUDA(cudaStreamSynchronize(s));
        if (code) return set_error(K3C_ETIMEOUT, "moe_decode_tc: device check code %d", code);
    }
    return K3C_OK;
}

}  // namespace k3c

extern "C" size_t k3c_pool_run_bytes(int hidden, int inter) {
    if (hidden <= 0 || inter <= 0 || hidden % 128 || inter % 128) return 0;
    return k3c::pool_geom(hidden, inter).run;
}

extern "C" int k3c_pool_pack_expert(uint8_t *run, const K3ExpertQ *src, int hidden, int inter,
                                    k3c_stream_t stream) {
    k3c::clear_error();
    if (!run || !src || hidden % 128 || inter % 128 || hidden <= 0 || inter <= 0)
        return k3c::set_error(K3C_EINVAL, "pool_pack: bad arguments (hidden=%d inter=%d)", hidden, inter);
    if (((uintptr_t)run & 255) || ((uintptr_t)src->p1 & 15) || ((uintptr_t)src->p2 & 15) || ((uintptr_t)src->p3 & 15))
        return k3c::set_error(K3C_EINVAL, "pool_pack: misaligned buffers");
    k3c::k_pool_pack<<<148 * 8, 256, 0, (cudaStream_t)stream>>>(run, *src, hidden, inter);
    K3C_CHECK_LAUNCH();
    return K3C_OK;
}

extern "C" size_t k3c_moe_decode_tc_scratch(const k3c_moe_pool_layer *L, int ntok) {
    return L ? k3c::moe_decode_tc_scratch(L, ntok) : 0;
}

extern "C" int k3c_moe_decode_tc_routed(float *out, const void *x, int x_dtype, int ntok,
                                        const k3c_moe_pool_layer *L, const int *idx, const float *wt, int *drops,
                                        void *scratch, size_t scratch_bytes, k3c_stream_t stream) {
    k3c::clear_error();
    return k3c::launch_moe_decode_tc(out, x, x_dtype, ntok, L, const_cast<int *>(idx), const_cast<float *>(wt),
                                     drops, scratch, scratch_bytes, (cudaStream_t)stream, true);
}

extern "C" int k3c_moe_decode_tc(float *out, const void *x, int x_dtype, int ntok,
                                 const k3c_moe_pool_layer *L, int *idx, float *wt, int *drops,
                                 void *scratch, size_t scratch_bytes, k3c_stream_t stream) {
    k3c::clear_error();
    return k3c::launch_moe_decode_tc(out, x, x_dtype, ntok, L, idx, wt, drops, scratch, scratch_bytes,
                                     (cudaStream_t)stream);
}
