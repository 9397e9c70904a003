/* A C consumer of libwdl_b200.so: compiled as C11 against include/wdl_b200.h and linked to the library, it calls
 * the host-only entry points (version, workspace sizes) and invalid calls that the library must reject before any
 * CUDA call, and prints what it saw. No GPU is needed: every call here returns before touching a device. */
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "wdl_b200.h"

#define FAKE ((void*)(uintptr_t)(1u << 20)) /* 256-byte aligned, checked but never dereferenced */

static int expect_argument_error(int status, const char* needle, const char* what) {
  if (status != WDL_ERR_ARGUMENT || strstr(wdl_last_error(), needle) == NULL) {
    printf("FAIL %s: status %d, message \"%s\"\n", what, status, wdl_last_error());
    return 1;
  }
  printf("ok %s: %s\n", what, wdl_last_error());
  return 0;
}

int main(void) {
  int failures = 0;
  printf("version %s\n", wdl_version());
  if (strncmp(wdl_version(), "wdl_b200", 8) != 0) failures++;
  size_t work = wdl_w4a4_linear_workspace(1392, 3072);
  printf("linear workspace %zu\n", work);
  if (work == 0 || work % 256 != 0) failures++;
  printf("sage prep workspace %zu\n", wdl_sage_prep_workspace(5568, 24));
  failures += expect_argument_error(
      wdl_w4a4_gemm(FAKE, FAKE, FAKE, FAKE, WDL_CODES_E4M3, NULL, 128, 300, 256, FAKE, 512, NULL), "multiple of 256",
      "gemm N % 256");
  failures += expect_argument_error(
      wdl_w4a4_gemm(FAKE, FAKE, FAKE, FAKE, 7, NULL, 128, 256, 256, FAKE, 256, NULL), "code format", "code format");
  failures += expect_argument_error(
      wdl_w4a4_linear(FAKE, 256, 128, 256, NULL, WDL_BF16, FAKE, FAKE, WDL_CODES_E4M3, NULL, 256, FAKE, 256, FAKE,
                      wdl_w4a4_linear_workspace(128, 256) - 1, NULL),
      "workspace", "linear workspace");
  /* a low-rank branch formed in the GEMM epilogue takes its rank in fours and a non-null activation */
  wdl_lowrank lr = {FAKE, 8, FAKE, 6};
  failures += expect_argument_error(
      wdl_w4a4_gemm_lowrank(FAKE, FAKE, FAKE, FAKE, WDL_CODES_E4M3, NULL, &lr, 128, 256, 256, FAKE, 256, NULL),
      "multiple of 4", "low-rank rank");
  lr.rank = 8;
  lr.act = NULL;
  failures += expect_argument_error(
      wdl_w4a4_gemm_residual_lowrank(FAKE, FAKE, FAKE, FAKE, WDL_CODES_E4M3, NULL, &lr, NULL, FAKE, 256, 128, 256, 256,
                                     FAKE, 256, NULL),
      "must not be null", "low-rank null act");
  if (wdl_w4a4_gemm(FAKE, FAKE, FAKE, FAKE, WDL_CODES_E4M3, NULL, 0, 256, 256, FAKE, 256, NULL) != WDL_OK) failures++;
  printf("%s\n", failures ? "FAILED" : "PASSED");
  return failures ? 1 : 0;
}
