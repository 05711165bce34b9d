/* A plain C (C99) caller of the library's C ABI, compiled and run by
 * tests/test_c_abi.py without a GPU. It checks that include/fa2_sm100.h is valid C, that the
 * struct layout the header describes matches the library's, and that the host-only entry
 * points (validation, workspace sizing, configuration, error strings) behave as documented.
 * It prints one line per check and exits non-zero on the first failure. */
#include <stdio.h>
#include <string.h>

#include "fa2_sm100.h"

static int fails = 0;
#define CHECK(cond, what)                                    \
  do {                                                       \
    if (cond) {                                              \
      printf("ok   %s\n", what);                             \
    } else {                                                 \
      printf("FAIL %s\n", what);                             \
      fails++;                                               \
    }                                                        \
  } while (0)

static void fill(Fa2FwdParams* p, int B, int Hq, int Hkv, int Nq, int Nkv, int D) {
  static char fake[64] __attribute__((aligned(16)));
  memset(p, 0, sizeof *p);
  p->q = p->k = p->v = fake; /* never dereferenced by the host-only calls below */
  p->o = fake;
  int64_t sq[4] = {(int64_t)Hq * Nq * D, (int64_t)Nq * D, D, 1};
  int64_t skv[4] = {(int64_t)Hkv * Nkv * D, (int64_t)Nkv * D, D, 1};
  memcpy(p->q_stride, sq, sizeof sq);
  memcpy(p->o_stride, sq, sizeof sq);
  memcpy(p->k_stride, skv, sizeof skv);
  memcpy(p->v_stride, skv, sizeof skv);
  p->batch = B;
  p->heads_q = Hq;
  p->heads_kv = Hkv;
  p->seqlen_q = Nq;
  p->seqlen_kv = Nkv;
  p->head_dim = D;
  p->dtype = FA2_DTYPE_BF16;
  p->causal = 1;
  p->qk_scale = 0.1275f;
}

int main(void) {
  Fa2FwdParams p;
  CHECK(fa2_sm100_abi_version() == FA2_SM100_ABI_VERSION, "ABI version matches the header");
  CHECK(fa2_sm100_params_size() == (int64_t)sizeof(Fa2FwdParams), "Fa2FwdParams size matches the library");

  fill(&p, 2, 32, 8, 8192, 8192, 128);
  CHECK(fa2_fwd_sm100_check(&p) == FA2_OK, "headline shape validates");
  CHECK(fa2_fwd_sm100_workspace_bytes(&p) == 0, "no split, no workspace");

  fill(&p, 2, 32, 8, 8192, 8192, 96);
  CHECK(fa2_fwd_sm100_check(&p) == FA2_ERR_HEAD_DIM, "head_dim 96 is rejected");
  fill(&p, 2, 32, 8, 1000, 1000, 32);
  CHECK(fa2_fwd_sm100_check(&p) == FA2_OK, "head_dim 32 runs in place on the 64 build");
  fill(&p, 2, 32, 8, 1000, 1000, 16);
  CHECK(fa2_fwd_sm100_check(&p) == FA2_OK, "head_dim 16 runs in place on the 64 build");
  fill(&p, 2, 30, 8, 8192, 8192, 128);
  CHECK(fa2_fwd_sm100_check(&p) == FA2_ERR_GQA, "H_q % H_kv != 0 is rejected");
  fill(&p, 2, 32, 8, 100, 200, 128);
  CHECK(fa2_fwd_sm100_check(&p) == FA2_ERR_SHAPE, "causal with N_q != N_kv is rejected");
  p.causal_align = FA2_CAUSAL_BOTTOM_RIGHT;
  CHECK(fa2_fwd_sm100_check(&p) == FA2_OK, "bottom-right causal accepts N_q < N_kv");
  fill(&p, 2, 32, 8, 300, 200, 128);
  p.causal_align = FA2_CAUSAL_BOTTOM_RIGHT;
  CHECK(fa2_fwd_sm100_check(&p) == FA2_ERR_SHAPE, "bottom-right causal rejects N_q > N_kv");
  fill(&p, 2, 32, 8, 8192, 8192, 128);
  p.q_stride[2] = 129; /* not a multiple of 8 elements */
  CHECK(fa2_fwd_sm100_check(&p) == FA2_ERR_LAYOUT, "unaligned stride is rejected");
  fill(&p, 2, 32, 8, 8192, 8192, 128);
  p.qk_scale = -1.0f;
  CHECK(fa2_fwd_sm100_check(&p) == FA2_ERR_SCALE, "negative qk_scale is rejected");
  CHECK(fa2_fwd_sm100_check(NULL) == FA2_ERR_NULL, "NULL params are rejected");

  fill(&p, 4, 32, 8, 1, 4096, 128);
  p.causal = 0;
  p.pack_gqa = 1;
  p.num_splits = 4;
  int64_t ws = fa2_fwd_sm100_workspace_bytes(&p);
  CHECK(ws > 0, "split-KV needs a workspace");
  CHECK(fa2_fwd_sm100_check(&p) == FA2_ERR_WORKSPACE, "split-KV without a workspace is rejected");

  int32_t bm = 0, bn = 0, th = 0, st = 0, sm = 0;
  CHECK(fa2_fwd_sm100_config(128, &bm, &bn, &th, &st, &sm) == FA2_OK && bm == 128 && bn == 128 && (th == 384 || th == 640) &&
            st >= 2 && sm > 0 && sm <= 227 * 1024,
        "config of the D=128 kernel");
  CHECK(fa2_fwd_sm100_config(80, &bm, &bn, &th, &st, &sm) == FA2_ERR_HEAD_DIM, "config rejects D=80");
  CHECK(strlen(fa2_sm100_strerror(FA2_ERR_LAYOUT)) > 0 && strcmp(fa2_sm100_strerror(FA2_OK), "ok") == 0,
        "error strings");
  printf("%s\n", fails ? "FAILED" : "ALL OK");
  return fails ? 1 : 0;
}
