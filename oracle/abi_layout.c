/* abi_layout.c -- prints sizeof/offsetof of the reference types that cross the drop-in
 * boundary (K3ExpertQ, K3ExpertSrc, K3Cfg, K3MoeW). TEST INFRASTRUCTURE ONLY.
 *
 * Built twice: against the reference's include/k3/k3.h (oracle/Makefile, into oracle/_ref/)
 * and against this repository's include/k3c.h (-DUSE_K3C, by tests/test_abi.py); the two
 * outputs must be identical for libk3cuda.so to be a drop-in for the reference's callers. */
#include <stddef.h>
#include <stdio.h>

#ifdef USE_K3C
#include "k3c.h"
#else
#include "k3.h"
#endif

#define F(T, m) printf("%s.%s %zu %zu\n", #T, #m, offsetof(T, m), sizeof(((T *)0)->m))
#define S(T) printf("%s %zu\n", #T, sizeof(T))

int main(void)
{
    S(K3ExpertQ);
    F(K3ExpertQ, p1); F(K3ExpertQ, s1); F(K3ExpertQ, p3); F(K3ExpertQ, s3); F(K3ExpertQ, p2); F(K3ExpertQ, s2);
    S(K3ExpertSrc);
    F(K3ExpertSrc, get); F(K3ExpertSrc, getmany); F(K3ExpertSrc, resident); F(K3ExpertSrc, ctx);
    S(K3Cfg);
    F(K3Cfg, hidden); F(K3Cfg, n_layers); F(K3Cfg, vocab); F(K3Cfg, rms_eps); F(K3Cfg, kda_heads);
    F(K3Cfg, kda_head_dim); F(K3Cfg, conv_k); F(K3Cfg, gate_lb); F(K3Cfg, n_heads); F(K3Cfg, q_lora);
    F(K3Cfg, kv_lora); F(K3Cfg, qk_nope); F(K3Cfg, qk_rope); F(K3Cfg, v_head); F(K3Cfg, mla_out_gate);
    F(K3Cfg, n_experts); F(K3Cfg, topk); F(K3Cfg, n_shared); F(K3Cfg, latent); F(K3Cfg, moe_inter);
    F(K3Cfg, routed_scale); F(K3Cfg, moe_renorm); F(K3Cfg, latent_norm); F(K3Cfg, first_dense);
    F(K3Cfg, dense_inter); F(K3Cfg, attn_res_block); F(K3Cfg, situ_b1); F(K3Cfg, situ_b2);
    F(K3Cfg, n_full_attn); F(K3Cfg, full_attn);
    S(K3MoeW);
    F(K3MoeW, gate); F(K3MoeW, bias); F(K3MoeW, w1); F(K3MoeW, w3); F(K3MoeW, w2); F(K3MoeW, latent_norm);
    F(K3MoeW, down); F(K3MoeW, up); F(K3MoeW, sh1); F(K3MoeW, sh3); F(K3MoeW, sh2); F(K3MoeW, wdt);
    F(K3MoeW, src); F(K3MoeW, layer); F(K3MoeW, cache_only);
    printf("K3_MXFP4_GROUP %d\nK3_MAX_TOPK %d\nK3_WF32 %d K3_WBF16 %d K3_WI8 %d\n", K3_MXFP4_GROUP, K3_MAX_TOPK,
           K3_WF32, K3_WBF16, K3_WI8);
    return 0;
}
