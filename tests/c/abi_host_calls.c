/* A C99 caller of include/bsattn.h: the calls that need no GPU (version, error text, workspace
 * size, argument checks that run before any device access, host-built work lists and CSR sizes).
 * Prints one line per check and "all ok" at the end; exits non-zero on the first mismatch. */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include "bsattn.h"

static int failures = 0;

static void expect(const char* what, long got, long want) {
  printf("%-44s %ld (want %ld)\n", what, got, want);
  if (got != want) ++failures;
}

int main(void) {
  char buf[16] __attribute__((aligned(16)));
  size_t bytes = 0;
  int32_t row_ptr[5] = {0, 1, 3, 5, 7}; /* 4 query blocks: diagonal, then previous + diagonal */
  int32_t plan[64];

  expect("bsattn_version", bsattn_version(), 102);
  expect("workspace bytes >= 4", bsattn_workspace_bytes() >= 4, 1);
  expect("strerror(E_NULL) is text", bsattn_strerror(BSATTN_E_NULL)[0] != '\0', 1);

  /* bsattn_fwd argument checks (no device access before them). */
  expect("fwd with q == NULL", bsattn_fwd(NULL, buf, buf, buf, NULL, (const int32_t*)buf,
                                          (const int32_t*)buf, NULL, 1, 1, 128, 128, 0, 0, 1,
                                          0.0f, BSATTN_OUT_F16, buf, 256, NULL),
         BSATTN_E_NULL);
  expect("fwd with D == 64", bsattn_fwd(buf, buf, buf, buf, NULL, (const int32_t*)buf,
                                        (const int32_t*)buf, NULL, 1, 1, 128, 64, 0, 0, 1,
                                        0.0f, BSATTN_OUT_F16, buf, 256, NULL),
         BSATTN_E_SHAPE);
  expect("fwd with T % 128 != 0", bsattn_fwd(buf, buf, buf, buf, NULL, (const int32_t*)buf,
                                             (const int32_t*)buf, NULL, 1, 1, 200, 128, 0, 0, 1,
                                             0.0f, BSATTN_OUT_F16, buf, 256, NULL),
         BSATTN_E_SHAPE);
  expect("fwd with an unknown dtype flag", bsattn_fwd(buf, buf, buf, buf, NULL,
                                                      (const int32_t*)buf, (const int32_t*)buf,
                                                      NULL, 1, 1, 128, 128, 0, 0, 1, 0.0f, 8,
                                                      buf, 256, NULL),
         BSATTN_E_DTYPE);
  expect("window with window == 0", bsattn_fwd_window(buf, buf, buf, buf, NULL, NULL, 1, 1, 128,
                                                      128, 0, 0, 0.0f, BSATTN_OUT_F16, NULL, 0,
                                                      buf, 256, NULL),
         BSATTN_E_SHAPE);

  /* Host-built work list: 4 items (T = 512) over 2 CTAs. */
  expect("plan_bytes rc", bsattn_plan_bytes(1, 1, 512, 2, &bytes), BSATTN_OK);
  expect("plan_bytes value", (long)bytes, (long)((4 + 3 + 4) * sizeof(int32_t)));
  expect("plan rc", bsattn_plan(row_ptr, 0, NULL, 1, 1, 512, 7, 2, plan, sizeof(plan)), BSATTN_OK);
  expect("plan header: grid", plan[1], 2);
  expect("plan header: items", plan[2], 4);
  expect("plan: CTA 0 + CTA 1 items", plan[4 + 2], 4);

  /* CSR sizes of the device-built families. */
  {
    int64_t nnz = 0;
    expect("csr_nnz rc (window 2, 4 rows)", bsattn_csr_nnz(BSATTN_CSR_WINDOW, 4, 0, 2, 0, &nnz),
           BSATTN_OK);
    expect("csr_nnz value", (long)nnz, 7);
  }

  if (failures) {
    printf("%d checks failed\n", failures);
    return 1;
  }
  printf("all ok\n");
  return 0;
}
