/*
 * A C99 caller of the library: includes the public header as plain C, links
 * against libw4a8moe.so and makes only calls that return before any device
 * work (version, workspace sizing, host-side argument checks), so it runs on
 * a machine without a GPU.  Built and run by tests/test_capi_c.py.
 */
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "w4a8moe.h"

#define FAKE(T) ((T)(uintptr_t)0x100000) /* never dereferenced: every call below fails validation first */

int main(void) {
  if (w4a8_abi_version() != 1) {
    printf("abi version %d\n", w4a8_abi_version());
    return 1;
  }
  if (w4a8_moe_align_workspace_size(16, 8, 256) < 4 * (256 + 128)) {
    printf("workspace too small\n");
    return 2;
  }
  /* group_size 96 does not divide K = 512: rejected on the host */
  int rc = w4a8_group_gemm_moe_ex(FAKE(const int8_t*), 512, FAKE(const float*), FAKE(const uint8_t*),
                                  FAKE(const float*), FAKE(const int8_t*), FAKE(const int32_t*), FAKE(void*), 512, 1,
                                  32, 4, 512, 512, 96, W4A8_KERNEL_AUTO, NULL, NULL);
  if (rc != W4A8_ERR_INVALID || strstr(w4a8_last_error(), "group_size") == NULL) {
    printf("expected a group_size error, got %d: %s\n", rc, w4a8_last_error());
    return 3;
  }
  /* nothing to do is not an error */
  rc = w4a8_group_gemm_moe_ex(FAKE(const int8_t*), 512, FAKE(const float*), FAKE(const uint8_t*), FAKE(const float*),
                              FAKE(const int8_t*), FAKE(const int32_t*), FAKE(void*), 512, 1, 0, 4, 512, 512, 128,
                              W4A8_KERNEL_AUTO, NULL, NULL);
  if (rc != W4A8_OK) {
    printf("empty call returned %d\n", rc);
    return 4;
  }
  printf("ok\n");
  return 0;
}
