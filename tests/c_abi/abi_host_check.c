/* A plain-C caller of libfast_trimul_b200: compiles against include/fast_trimul_b200.h
 * alone and exercises the host-side part of the boundary -- sizes, status strings and
 * argument checks, which return before any device call. Prints one line per check and
 * exits non-zero on the first mismatch. Run by tests/test_api_cpu.py. */
#include <stdio.h>
#include <string.h>

#include "fast_trimul_b200.h"

static int fails = 0;
#define CHECK(cond, what)                                   \
  do {                                                      \
    if (!(cond)) {                                          \
      printf("FAIL %s\n", what);                            \
      ++fails;                                              \
    } else {                                                \
      printf("ok   %s\n", what);                            \
    }                                                       \
  } while (0)

int main(void) {
  ftm_problem p;
  memset(&p, 0, sizeof(p));
  p.batch = 1; p.rows = 256; p.cols = 256; p.c_z = 128; p.c_h = 128;
  p.mode = FTM_OUTGOING; p.residual = 1; p.z_dtype = FTM_BF16; p.out_dtype = FTM_BF16;
  p.eps_in = 1e-5f; p.eps_out = 1e-5f;

  CHECK(ftm_packed_params_bytes(128, 128) > 0, "packed parameter size");
  /* three fp16 planes of B * c_h * N^2 plus statistics and the error word */
  CHECK(ftm_workspace_bytes(&p) >= (size_t)3 * 128 * 256 * 256 * 2, "workspace size");
  CHECK(strcmp(ftm_status_string(FTM_OK), "ok") == 0, "status string");

  ftm_problem bad = p;
  bad.c_z = 64;
  CHECK(ftm_workspace_bytes(&bad) == 0, "unsupported width has no workspace");
  bad = p;
  bad.cols = 250;
  CHECK(ftm_trimul_fwd(&bad, (void*)16, NULL, (void*)16, (void*)16, (void*)16, 1 << 30, NULL) ==
            FTM_BAD_SHAPE, "N % 8 rejected");
  CHECK(ftm_trimul_fwd(NULL, NULL, NULL, NULL, NULL, NULL, 0, NULL) != FTM_OK, "null problem");
  CHECK(ftm_contraction_kblocked((void*)16, (void*)16, (void*)16, 3, 512, 512, 100, 2, 256, NULL,
                                 NULL) != FTM_OK, "k block size rejected");

  ftm_peer_planes planes;
  memset(&planes, 0, sizeof(planes));
  planes.world = 3;   /* 128 channels do not split over 3 ranks */
  planes.rank = 0;
  planes.base[0] = (void*)16; planes.base[1] = (void*)32; planes.base[2] = (void*)48;
  CHECK(ftm_input_stage_scatter(&p, (void*)16, NULL, (void*)16, &planes, &planes, (float*)16,
                                (int*)16, NULL) == FTM_BAD_ARGUMENT, "uneven channel split");
  printf("%s\n", fails ? "FAILED" : "all host-side checks passed");
  return fails ? 1 : 0;
}
