// moe_tc.cu -- MoE decode on the 5th-generation tensor cores (tcgen05, kind::mxf8f6f4).
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

namespace k3c {

int launch_router_scores(float *scores, const void *x, int x_dtype, const void *W, int w_dtype,
                         int hidden, int n_experts, int ntok, cudaStream_t s);
int launch_router_select(int *idx, float *w, const float *scores, const float *bias,
                         int n_experts, int topk, int renorm, float routed_scale, int ntok,
                         cudaStream_t s);
int launch_moe_combine(float *out, const float *contrib, const float *wt, const uint8_t *dropped,
                       int ntok, int topk, int hidden, int has_shared, cudaStream_t s);

struct PoolGeom {
    size_t gu_p, gu_s, d_p, d_s, run;
};
__host__ __device__ inline PoolGeom pool_geom(int H, int I) {
    PoolGeom g;
    g.gu_p = 0;
    g.gu_s = (size_t)I * H;                                // 2I rows x H/2 bytes
    g.d_p = g.gu_s + (size_t)(2 * I / 128) * (H / 128) * 512;
    g.d_s = g.d_p + (size_t)H * I / 2;
    g.run = g.d_s + (size_t)(H / 128) * (I / 128) * 512;
    return g;
}

// GU row R -> (source matrix: 0 gate / 1 up, source row).
__host__ __device__ inline void gu_source(int R, int &which, int &row) {
    const int b = R / 128, m = R % 128;
    which = m >= 64;
    row = 64 * b + (m & 63);
}

__device__ __forceinline__ size_t atom_byte(int m, int g) {  // m: row in tile, g: group 0..3
    return (size_t)(16 * (m & 31) + 4 * (m >> 5) + g);
}

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
// Block exponent e for a block maximum amax so that amax / 2^e <= 448 (the E4M3 maximum):
// e = ceil(log2(amax / 448)), clamped to the UE8M0 range used here [-127, 120].
__device__ __forceinline__ int block_exp(float amax) {
    const uint32_t u = __float_as_uint(amax);
    const int E = (int)((u >> 23) & 0xFF) - 127;
    if (amax == 0.0f || E < -119) return -127;
    int e = ((u & 0x7FFFFF) > 0x600000) ? E - 7 : E - 8;  // mantissa > 1.75 -> one more
    return e < -127 ? -127 : (e > 120 ? 120 : e);
}
__device__ __forceinline__ float exp2i(int e) {  // 2^e, e in [-126, 127]
    return __uint_as_float((uint32_t)(e + 127) << 23);
}

// One warp quantises one 32-element block held one element per lane into J terms.
// Writes each term's byte through qdst(j) and its scale byte through sfdst(j) (lane 0).
template <int J, class QF, class SF>
__device__ __forceinline__ void quantize_block(float a, QF qdst, SF sfdst) {
#pragma unroll
    for (int j = 0; j < J; j++) {
        float amax = fabsf(a);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const int e = block_exp(amax);                 // e in [-127, 120]
        const uint32_t q = tc::f32_to_e4m3(a * exp2i(-e)); // 2^-e in [2^-120, 2^127]: exact
        qdst(j, q);
        if ((threadIdx.x & 31) == 0) sfdst(j, (uint32_t)(e + 127));
        const float back = tc::e4m3_to_f32(q);
        // back * 2^e exactly; 2^-127 is formed as 2^-126 / 2
        a = a - (e >= -126 ? back * exp2i(e) : (back * exp2i(-126)) * 0.5f);
    }
}

// x [ntok][H] -> x_q [J][32][H] E4M3 and x_sf [J][H/128] atoms (rows = tokens, < 32).
template <int J, typename XT>
__global__ void __launch_bounds__(256) k_quant_x(uint8_t *__restrict__ xq, uint8_t *__restrict__ xsf,
                                                 const XT *__restrict__ x, int ntok, int H) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int blk = blockIdx.x * 8 + warp;  // 32-element block index
    const int t = blockIdx.y;
    if (blk * 32 >= H || t >= ntok) return;
    const int k = blk * 32 + lane;
    float a;
    if constexpr (sizeof(XT) == 2) a = bf16_bits_to_f32(x[(size_t)t * H + k]);
    else a = x[(size_t)t * H + k];
    const int KT = H / 128;
    quantize_block<J>(
        a, [&](int j, uint32_t q) { xq[((size_t)j * 32 + t) * H + k] = (uint8_t)q; },
        [&](int j, uint32_t sf) {
            xsf[((size_t)j * KT + blk / 4) * 512 + atom_byte(t, blk % 4)] = (uint8_t)sf;
        });
}

// ------------------------------------------------------------------ plan (tc)
struct SlotTc {
    int run, ntok;
};

// Same grouping as the CUDA-core plan, slot-major with 32 pair rows per slot.
__global__ void __launch_bounds__(1024) k_moe_plan_tc(int *__restrict__ n_slots, SlotTc *__restrict__ slots,
                                                      int *__restrict__ pair_tok, int *__restrict__ pair_k,
                                                      uint8_t *__restrict__ dropped, const int *__restrict__ idx,
                                                      int ntok, int topk, const int *__restrict__ run_of,
                                                      int n_experts, int n_runs, int shared_run,
                                                      int *__restrict__ drops) {
    extern __shared__ int sm[];
    int *cnt = sm, *slot_of = sm + n_experts;
    const int P = ntok * topk;
    for (int e = threadIdx.x; e < n_experts; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < P; i += blockDim.x) {
        const int e = idx[i];
        // a run index outside the arena is treated as not resident: the kernels form raw
        // scale addresses from it
        const bool ok = e >= 0 && e < n_experts && run_of[e] >= 0 && run_of[e] < n_runs;
        dropped[i] = ok ? 0 : 1;
        if (ok) atomicAdd(&cnt[e], 1);
        else if (drops) atomicAdd(drops, 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int ns = 0;
        for (int e = 0; e < n_experts; e++) {
            if (cnt[e] > 0) {
                slot_of[e] = ns;
                slots[ns].run = run_of[e];
                slots[ns].ntok = cnt[e];
                ns++;
            } else {
                slot_of[e] = -1;
            }
        }
        if (shared_run >= 0) {
            slots[ns].run = shared_run;
            slots[ns].ntok = ntok;
            for (int t = 0; t < ntok; t++) {
                pair_tok[ns * 32 + t] = t;
                pair_k[ns * 32 + t] = topk;
            }
            ns++;
        }
        *n_slots = ns;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < P; i += blockDim.x) {
        if (dropped[i]) continue;
        const int e = idx[i];
        int rank = 0;
        for (int k = 0; k < i; k++) rank += (idx[k] == e && !dropped[k]);
        const int pos = slot_of[e] * 32 + rank;
        pair_tok[pos] = i / topk;
        pair_k[pos] = i % topk;
    }
}

// ------------------------------------------------------------------ tcgen05 mainloop
constexpr int TC_NT = 32;           // N tile: tokens (GU) or pairs of a slot (D)
constexpr int TC_A_BYTES = 128 * 128;   // shared-memory footprint of a padded E2M1 tile
constexpr int TC_A_TX = 128 * 128 / 2;  // its TMA transaction bytes: 4 bits per element
constexpr int TC_B_BYTES = TC_NT * 128;
constexpr uint32_t TC_TMEM_COLS = 64;

template <int J, int STAGES>
struct TcSmem {
    static constexpr int STAGE = TC_A_BYTES + J * TC_B_BYTES + 512 + J * 512;
    static constexpr int BYTES = STAGES * STAGE + 1024 /* align */ + 256 /* barriers */;
};

struct TcArgs {
    const int *n_slots;
    const SlotTc *slots;
    const int *pair_tok, *pair_k;
    const uint8_t *arena;
    size_t run_stride;
    const uint8_t *b_sf;     // GU activation scale atoms [J][H/128][512] (tokens = atom rows 0..31)
    uint8_t *act_q;          // GU output: [J][S*32][I], slot s owns rows 32s..32s+31
    uint8_t *act_sf;         // GU output atoms [J][S][I/128][512], one atom per slot (rows 0..31)
    int act_slots;           // S
    float *contrib;          // D output [T][topk+1][H]
    int kstride;             // topk + 1
    int H, I, act;
    int *err;
};

// Stage layout inside one pipeline stage: A | B[J] | SFA | SFB[J].
template <int J>
struct StagePtr {
    uint8_t *a, *b[J], *sfa, *sfb[J];
    __device__ StagePtr(uint8_t *base) {
        a = base;
#pragma unroll
        for (int j = 0; j < J; j++) b[j] = base + TC_A_BYTES + j * TC_B_BYTES;
        sfa = base + TC_A_BYTES + J * TC_B_BYTES;
#pragma unroll
        for (int j = 0; j < J; j++) sfb[j] = sfa + 512 + j * 512;
    }
};

// Runs the K loop for one M=128 x N=32 tile: warp 0 lane 0 produces (TMA), warp 1 lane 0
// issues tcgen05 copies and MMAs; returns with the accumulator in TMEM columns [0,32) and
// the accum barrier armed. kt_count: K tiles of 128. a_* select the weight tile, b_row the
// activation rows (whose scales sit in rows 0..31 of their atoms).
// Alignment self-checks: a violated precondition records an error code in *err and the
// loop stops issuing, instead of handing the hardware a misaligned address.
__device__ __forceinline__ bool tc_check(bool ok, int *err, int code) {
    if (!ok && err) atomicExch(err, code);
    return ok;
}

template <int J, int STAGES>
__device__ __forceinline__ void tc_mainloop(uint8_t *smem, uint64_t *full, uint64_t *empty,
                                            uint64_t *accum, uint32_t tmem, const CUtensorMap *tmA,
                                            const CUtensorMap *tmB, const uint8_t *sfa_base,
                                            const uint8_t *sfb_base, size_t sfb_term_stride,
                                            int a_row, int a_run, int b_row, int kt_count, int *err) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int STAGE = TcSmem<J, STAGES>::STAGE;
    if (warp == 0 && lane == 0) {
        if (!tc_check(((uintptr_t)sfa_base & 15) == 0 && ((uintptr_t)sfb_base & 15) == 0 &&
                          (sfb_term_stride & 15) == 0 && (tc::smem_u32(smem) & 1023) == 0,
                      err, 10))
            return;
        tc::prefetch_tmap(tmA);
        tc::prefetch_tmap(tmB);
        for (int kt = 0; kt < kt_count; kt++) {
            const int st = kt % STAGES;
            const uint32_t ph = (uint32_t)(kt / STAGES) & 1u;
            if (kt >= STAGES && !tc::mbar_wait(&empty[st], ph ^ 1u, err, 1)) return;
            StagePtr<J> sp(smem + st * STAGE);
            tc::mbar_expect_tx(&full[st], TC_A_TX + 512 + J * (TC_B_BYTES + 512));
            tc::tma_load_3d(sp.a, tmA, &full[st], kt * 128, a_row, a_run);
            tc::bulk_load(sp.sfa, sfa_base + (size_t)kt * 512, 512, &full[st]);
#pragma unroll
            for (int j = 0; j < J; j++) {
                tc::tma_load_3d(sp.b[j], tmB, &full[st], kt * 128, b_row, j);
                tc::bulk_load(sp.sfb[j], sfb_base + j * sfb_term_stride + (size_t)kt * 512, 512, &full[st]);
            }
        }
    } else if (warp == 1 && lane == 0) {
        for (int kt = 0; kt < kt_count; kt++) {
            const int st = kt % STAGES;
            const uint32_t ph = (uint32_t)(kt / STAGES) & 1u;
            if (!tc::mbar_wait(&full[st], ph, err, 2)) return;
            tc::tc_fence_after();
            StagePtr<J> sp(smem + st * STAGE);
            const uint32_t sf_col = 32u + 16u * (uint32_t)(kt & 1);  // double-buffered
            tc::tc_cp_sf(tmem + sf_col, tc::desc_sf_atom(tc::smem_u32(sp.sfa)));
#pragma unroll
            for (int j = 0; j < J; j++)
                tc::tc_cp_sf(tmem + sf_col + 4 + 4 * j, tc::desc_sf_atom(tc::smem_u32(sp.sfb[j])));
#pragma unroll
            for (int kb = 0; kb < 4; kb++) {
                const uint64_t da = tc::desc_kmajor_sw128(tc::smem_u32(sp.a) + 32 * kb);
#pragma unroll
                for (int j = 0; j < J; j++) {
                    const uint64_t db = tc::desc_kmajor_sw128(tc::smem_u32(sp.b[j]) + 32 * kb);
                    const uint32_t id = tc::idesc_mxf8f6f4(tc::FMT_E2M1, tc::FMT_E4M3, TC_NT, kb, kb);
                    const uint32_t sfa = (tmem + sf_col) | ((uint32_t)kb << 30);
                    const uint32_t sfb = (tmem + sf_col + 4 + 4 * j) | ((uint32_t)kb << 30);
                    tc::tc_mma_mx(tmem, da, db, id, sfa, sfb, (kt | kb | j) != 0);
                }
            }
            tc::tc_commit(&empty[st]);
        }
        tc::tc_commit(accum);
    }
}

__device__ __forceinline__ float sigmoid_f(float v) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v))); }
__device__ __forceinline__ float act_apply(float g, float u, int act) {
    if (act == K3C_ACT_SITU) {
        const float a = __fmul_rn(__fmul_rn(4.0f, tanhf(__fdiv_rn(g, 4.0f))), sigmoid_f(g));
        return __fmul_rn(a, __fmul_rn(25.0f, tanhf(__fdiv_rn(u, 25.0f))));
    }
    return __fmul_rn(__fmul_rn(g, sigmoid_f(g)), u);
}

// Shared prologue: barriers + TMEM; returns the TMEM base.
template <int STAGES>
__device__ __forceinline__ uint32_t tc_setup(uint64_t *bars, uint32_t *tmem_slot) {
    const int warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        for (int i = 0; i < 2 * STAGES + 1; i++) tc::mbar_init(&bars[i], 1);
        tc::fence_mbar_init();
    }
    if (warp == 1) tc::tmem_alloc(tmem_slot, TC_TMEM_COLS);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    return *tmem_slot;
}

template <int STAGES>
__device__ __forceinline__ void tc_teardown(uint32_t tmem) {
    tc::tc_fence_before();
    __syncthreads();
    if ((threadIdx.x >> 5) == 1) tc::tmem_dealloc(tmem, TC_TMEM_COLS);
}

// GU stage: grid (2I/128, max_slots), 128 threads. Tile rows: 64 gate + 64 up rows of output
// columns [64*bx, 64*bx+64); N = 32 token columns (all tokens; the slot's pairs pick theirs).
template <int J, int STAGES>
__global__ void __launch_bounds__(128) k_tc_gateup(const __grid_constant__ CUtensorMap tmW,
                                                   const __grid_constant__ CUtensorMap tmX, TcArgs p) {
    const int s = blockIdx.y;
    if (s >= *p.n_slots) return;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    constexpr int STAGE = TcSmem<J, STAGES>::STAGE;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE);
    uint64_t *full = bars, *empty = bars + STAGES, *accum = bars + 2 * STAGES;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * STAGES + 1);
    const uint32_t tmem = tc_setup<STAGES>(bars, tmem_slot);

    const SlotTc sl = p.slots[s];
    const int rt = blockIdx.x, KT = p.H / 128;
    const PoolGeom g = pool_geom(p.H, p.I);
    const uint8_t *run = p.arena + (size_t)sl.run * p.run_stride;
    tc_mainloop<J, STAGES>(smem, full, empty, accum, tmem, &tmW, &tmX,
                           run + g.gu_s + (size_t)rt * KT * 512, p.b_sf, (size_t)KT * 512,
                           rt * 128, sl.run, 0, KT, p.err);
    __syncwarp();
    const bool ok = tc::mbar_wait(accum, 0, p.err, 3);
    tc::tc_fence_after();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float *tile = reinterpret_cast<float *>(smem);  // [128][33], reuses stage 0
    if (ok) {
        uint32_t v[32];
        tc::tmem_ld32(tmem + ((uint32_t)(32 * warp) << 16), v);
        tc::tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 32; c++) tile[(32 * warp + lane) * 33 + c] = __uint_as_float(v[c]);
    }
    __syncthreads();
    if (ok && warp < 2) {
        const int r = 32 * warp + lane;               // gate row within the tile
        const int col = 64 * rt + r;                  // output column in [0, I)
        const int KTd = p.I / 128;
        for (int pl = 0; pl < sl.ntok; pl++) {
            const int prow = s * 32 + pl;
            const int tok = p.pair_tok[prow];
            const float a = act_apply(tile[r * 33 + tok], tile[(r + 64) * 33 + tok], p.act);
            quantize_block<J>(
                a,
                [&](int j, uint32_t q) {
                    p.act_q[((size_t)j * p.act_slots * 32 + prow) * p.I + col] = (uint8_t)q;
                },
                [&](int j, uint32_t sf) {
                    const size_t atom = ((size_t)j * p.act_slots + s) * KTd + col / 128;
                    p.act_sf[atom * 512 + atom_byte(pl, (col % 128) / 32)] = (uint8_t)sf;
                });
        }
    }
    tc_teardown<STAGES>(tmem);
}

// D stage: grid (H/128, max_slots). A = down rows [128*bx, +128), B = the slot's 32 pair rows
// of act_q. Epilogue writes the unweighted expert output for each pair to contrib.
template <int J, int STAGES>
__global__ void __launch_bounds__(128) k_tc_down(const __grid_constant__ CUtensorMap tmW,
                                                 const __grid_constant__ CUtensorMap tmA, TcArgs p) {
    const int s = blockIdx.y;
    if (s >= *p.n_slots) return;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    constexpr int STAGE = TcSmem<J, STAGES>::STAGE;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE);
    uint64_t *full = bars, *empty = bars + STAGES, *accum = bars + 2 * STAGES;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * STAGES + 1);
    const uint32_t tmem = tc_setup<STAGES>(bars, tmem_slot);

    const SlotTc sl = p.slots[s];
    const int rt = blockIdx.x, KT = p.I / 128;
    const PoolGeom g = pool_geom(p.H, p.I);
    const uint8_t *run = p.arena + (size_t)sl.run * p.run_stride;
    const uint8_t *sfb = p.act_sf + (size_t)s * KT * 512;
    tc_mainloop<J, STAGES>(smem, full, empty, accum, tmem, &tmW, &tmA,
                           run + g.d_s + (size_t)rt * KT * 512, sfb, (size_t)p.act_slots * KT * 512,
                           rt * 128, sl.run, s * 32, KT, p.err);
    __syncwarp();
    const bool ok = tc::mbar_wait(accum, 0, p.err, 3);
    tc::tc_fence_after();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (ok) {
        uint32_t v[32];
        tc::tmem_ld32(tmem + ((uint32_t)(32 * warp) << 16), v);
        tc::tmem_ld_wait();
        const int h = 128 * rt + 32 * warp + lane;
#pragma unroll
        for (int pl = 0; pl < 32; pl++) {
            if (pl < sl.ntok) {
                const int prow = s * 32 + pl;
                p.contrib[((size_t)p.pair_tok[prow] * p.kstride + p.pair_k[prow]) * p.H + h] =
                    __uint_as_float(v[pl]);
            }
        }
    }
    tc_teardown<STAGES>(tmem);
}

// ------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

static int make_map3(CUtensorMap *m, CUtensorMapDataType dt, const void *base, uint64_t d0, uint64_t d1,
                     uint64_t d2, uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return set_error(K3C_ECUDA, "tc: cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[3] = {d0, d1, d2}, strides[2] = {s1, s2};
    cuuint32_t box[3] = {b0, b1, 1}, es[3] = {1, 1, 1};
    CUresult r = fn(m, dt, 3, const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(K3C_ECUDA, "tc: tensor map encode failed (%d)", (int)r);
    return K3C_OK;
}

struct TcBufs {
    int *n_slots;
    SlotTc *slots;
    int *pair_tok, *pair_k;
    uint8_t *dropped;
    float *scores, *wt, *contrib;
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
    b.err = cv.take<int>(1);
    b.slots = cv.take<SlotTc>(b.max_slots);
    b.pair_tok = cv.take<int>((size_t)b.max_slots * 32);
    b.pair_k = cv.take<int>((size_t)b.max_slots * 32);
    b.dropped = cv.take<uint8_t>(P);
    b.scores = cv.take<float>((size_t)ntok * L->n_experts);
    b.idx = cv.take<int>(P);
    b.wt = cv.take<float>(P);
    b.contrib = cv.take<float>((size_t)ntok * (L->topk + 1) * H);
    b.xq = cv.take<uint8_t>((size_t)J * 32 * H, 1024);
    b.xsf = cv.take<uint8_t>((size_t)J * (H / 128) * 512, 1024);
    b.actq = cv.take<uint8_t>((size_t)J * b.max_slots * 32 * I, 1024);
    b.actsf = cv.take<uint8_t>((size_t)J * b.max_slots * (I / 128) * 512, 1024);
    return b.n_slots && b.err && b.slots && b.pair_tok && b.pair_k && b.dropped && b.scores &&
           b.idx && b.wt && b.contrib && b.xq && b.xsf && b.actq && b.actsf;
}

static char *const kSizing = reinterpret_cast<char *>(4096);

size_t moe_decode_tc_scratch(const k3c_moe_pool_layer *L, int ntok) {
    Carve cv{kSizing, (size_t)-1 / 2, 0};
    TcBufs b;
    carve_tc(cv, b, L, ntok);
    return cv.used + 1024;
}

template <int J, int STAGES>
static int launch_tc_stages(const TcBufs &b, const k3c_moe_pool_layer *L, int ntok, cudaStream_t s) {
    const int H = L->hidden, I = L->inter;
    const PoolGeom g = pool_geom(H, I);
    CUtensorMap tmGU, tmD, tmX, tmAct;
    K3C_TRY(make_map3(&tmGU, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, L->arena + g.gu_p, H, 2 * I, L->n_runs,
                      H / 2, L->run_stride, 128, 128));
    K3C_TRY(make_map3(&tmD, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, L->arena + g.d_p, I, H, L->n_runs, I / 2,
                      L->run_stride, 128, 128));
    K3C_TRY(make_map3(&tmX, CU_TENSOR_MAP_DATA_TYPE_UINT8, b.xq, H, 32, J, H, (uint64_t)32 * H, 128, 32));
    K3C_TRY(make_map3(&tmAct, CU_TENSOR_MAP_DATA_TYPE_UINT8, b.actq, I, (uint64_t)b.max_slots * 32, J, I,
                      (uint64_t)b.max_slots * 32 * I, 128, 32));
    TcArgs a;
    a.n_slots = b.n_slots;
    a.slots = b.slots;
    a.pair_tok = b.pair_tok;
    a.pair_k = b.pair_k;
    a.arena = L->arena;
    a.run_stride = L->run_stride;
    a.b_sf = b.xsf;
    a.act_q = b.actq;
    a.act_sf = b.actsf;
    a.act_slots = b.max_slots;
    a.contrib = b.contrib;
    a.kstride = L->topk + 1;
    a.H = H;
    a.I = I;
    a.act = L->act;
    a.err = b.err;
    const int smem = TcSmem<J, STAGES>::BYTES;
    K3C_TRY_CUDA(cudaFuncSetAttribute(k_tc_gateup<J, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    K3C_TRY_CUDA(cudaFuncSetAttribute(k_tc_down<J, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    stage_begin(STAGE_EXPERTS, s);
    k_tc_gateup<J, STAGES><<<dim3(2 * I / 128, b.max_slots), 128, smem, s>>>(tmGU, tmX, a);
    K3C_CHECK_LAUNCH();
    k_tc_down<J, STAGES><<<dim3(H / 128, b.max_slots), 128, smem, s>>>(tmD, tmAct, a);
    K3C_CHECK_LAUNCH();
    stage_end(STAGE_EXPERTS, s);
    return K3C_OK;
}

int launch_moe_decode_tc(float *out, const void *x, int x_dtype, int ntok, const k3c_moe_pool_layer *L,
                         int *idx_out, float *wt_out, int *drops, void *scratch, size_t scratch_bytes,
                         cudaStream_t s) {
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
    K3C_TRY_CUDA(cudaMemsetAsync(b.err, 0, sizeof(int), s));
    stage_begin(STAGE_ROUTER, s);
    K3C_TRY(launch_router_scores(b.scores, x, x_dtype, L->router_w, L->router_dtype, H, L->n_experts, ntok, s));
    K3C_TRY(launch_router_select(idx, wt, b.scores, L->router_bias, L->n_experts, L->topk, L->renorm,
                                 L->routed_scale, ntok, s));
    stage_end(STAGE_ROUTER, s);
    const size_t psmem = (size_t)L->n_experts * 2 * sizeof(int);
    if (psmem > 48 * 1024)
        K3C_TRY_CUDA(cudaFuncSetAttribute(k_moe_plan_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)psmem));
    k_moe_plan_tc<<<1, 1024, psmem, s>>>(b.n_slots, b.slots, b.pair_tok, b.pair_k, b.dropped, idx, ntok,
                                         L->topk, L->run_of, L->n_experts, L->n_runs, L->shared_run, drops);
    K3C_CHECK_LAUNCH();
    dim3 gq(H / 256 + (H % 256 ? 1 : 0), ntok);
    switch (L->terms) {
    case 1:
        if (x_dtype == K3C_BF16) k_quant_x<1, uint16_t><<<gq, 256, 0, s>>>(b.xq, b.xsf, (const uint16_t *)x, ntok, H);
        else k_quant_x<1, float><<<gq, 256, 0, s>>>(b.xq, b.xsf, (const float *)x, ntok, H);
        K3C_CHECK_LAUNCH();
        K3C_TRY((launch_tc_stages<1, 4>(b, L, ntok, s)));
        break;
    case 2:
        if (x_dtype == K3C_BF16) k_quant_x<2, uint16_t><<<gq, 256, 0, s>>>(b.xq, b.xsf, (const uint16_t *)x, ntok, H);
        else k_quant_x<2, float><<<gq, 256, 0, s>>>(b.xq, b.xsf, (const float *)x, ntok, H);
        K3C_CHECK_LAUNCH();
        K3C_TRY((launch_tc_stages<2, 4>(b, L, ntok, s)));
        break;
    default:
        if (x_dtype == K3C_BF16) k_quant_x<3, uint16_t><<<gq, 256, 0, s>>>(b.xq, b.xsf, (const uint16_t *)x, ntok, H);
        else k_quant_x<3, float><<<gq, 256, 0, s>>>(b.xq, b.xsf, (const float *)x, ntok, H);
        K3C_CHECK_LAUNCH();
        K3C_TRY((launch_tc_stages<3, 3>(b, L, ntok, s)));
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

extern "C" int k3c_moe_decode_tc(float *out, const void *x, int x_dtype, int ntok,
                                 const k3c_moe_pool_layer *L, int *idx, float *wt, int *drops,
                                 void *scratch, size_t scratch_bytes, k3c_stream_t stream) {
    k3c::clear_error();
    return k3c::launch_moe_decode_tc(out, x, x_dtype, ntok, L, idx, wt, drops, scratch, scratch_bytes,
                                     (cudaStream_t)stream);
}
