/* A plain C consumer of the C ABI, compiled with gcc against include/moe_b200.h
 * and linked to the built library: checks the ABI version and the argument
 * validation of a few entry points, none of which launches a kernel, so it
 * runs on a host without a GPU. Exit status 0 on success. */
#include <stdio.h>
#include <string.h>

#include "moe_b200.h"

static int failures = 0;

static void expect(int cond, const char* what) {
  if (!cond) {
    fprintf(stderr, "FAIL: %s (last error: %s)\n", what, moe_b200_last_error());
    ++failures;
  }
}

int main(void) {
  size_t n = 0;
  expect(moe_b200_abi_version() == 2, "abi version");
  expect(moe_row_id_map_workspace_size(16384, 256, &n) == MOE_OK && n > 0, "rim workspace size");
  expect(moe_grouped_gemm_workspace_size(256, &n) == MOE_OK && n >= 256, "gemm workspace size");
  expect(moe_grouped_gemm_workspace_size(0, &n) == MOE_ERR_INVALID, "gemm workspace G=0");
  expect(moe_topk_f32((const float*)16, (float*)16, (int64_t*)16, 4, 64, 17, 0) ==
             MOE_ERR_UNSUPPORTED,
         "topk k=17");
  expect(moe_permute_mask_map(0, 0, 0, 0, 0, 0, 8, 2, 0, 0) == MOE_OK, "empty permute");
  expect(moe_swiglu_backward(0, 0, 0, 4, 12, 0) == MOE_ERR_INVALID, "swiglu_backward F=12");
  expect(strstr(moe_b200_last_error(), "multiple of 8") != NULL, "error text");
  if (failures == 0) printf("C consumer OK\n");
  return failures == 0 ? 0 : 1;
}
