/* Plain-C caller of liblp_b200.so through include/lp_logprob.h, as a cgo / JNI / ctypes
 * binding would call it. No GPU is needed: it checks the version, the workspace sizing
 * functions and that argument errors come back as LP_EINVAL with a message, before any
 * device work. Exit status 0 = all checks passed. */
#include <stdio.h>
#include <string.h>

#include "lp_logprob.h"

static int failures = 0;

static void expect(int cond, const char* what) {
  if (!cond) {
    fprintf(stderr, "FAIL: %s (last error: %s)\n", what, lp_last_error());
    ++failures;
  }
}

int main(void) {
  void* fake = (void*)(size_t)16; /* never dereferenced: every call below fails its checks */
  expect(lp_version() >= 100, "lp_version");
  expect(lp_fwd_workspace_bytes(0, 10) > 0, "lp_fwd_workspace_bytes on an empty batch");
  expect(lp_bwd_sum_counters(257) == 5, "lp_bwd_sum_counters: one per 128 rows + 2");
  expect(lp_compact_workspace_bytes(2, 3) > 0, "lp_compact_workspace_bytes");

  int rc = lp_fwd(NULL, fake, 4, 7, 7, fake, 10, 0, fake, 0.0f, fake, fake, fake, 1 << 20);
  expect(rc == LP_EINVAL && strstr(lp_last_error(), "multiple of 8") != NULL, "lp_fwd rejects d % 8 != 0");
  rc = lp_bwd(NULL, fake, 4, 8, 8, fake, 10, 0, fake, 0.0f, fake, fake, NULL, 8, fake, 0, 0, fake, 1 << 20);
  expect(rc == LP_EINVAL && strstr(lp_last_error(), "dH") != NULL, "lp_bwd requires dH");
  rc = lp_combine(NULL, fake, 0, 5, fake, fake);
  expect(rc == LP_EINVAL, "lp_combine rejects P = 0");
  rc = lp_head(NULL, fake, 4, 8, 8, fake, 10, 0.0f, fake, 9, 0, fake, NULL, NULL, fake, 1024);
  expect(rc == LP_EINVAL && strstr(lp_last_error(), "ld_logits") != NULL, "lp_head rejects ld_logits < V");
  rc = lp_fwd_sum(NULL, fake, 4, 8, 8, fake, 10, 0, fake, 0.0f, fake, fake, 4, fake, fake, fake, 0, 0, 2, 100, fake,
                  fake, fake, 1 << 20);
  expect(rc == LP_EINVAL && strstr(lp_last_error(), "epoch") != NULL, "lp_fwd_sum rejects epoch 0");
  rc = lp_fwd_noalloc(NULL, fake, 2000000, 64, 64, fake, 64, 0, fake, 0.0f, fake, NULL);
  expect(rc == LP_EINVAL || rc == LP_ECUDA || rc == LP_EUNSUPPORTED, "lp_fwd_noalloc refuses without device work");
  expect(lp_set_cta_group(3) == LP_EINVAL, "lp_set_cta_group rejects 3");
  if (failures == 0) printf("c abi smoke: ok\n");
  return failures == 0 ? 0 : 1;
}
