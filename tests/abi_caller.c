/* A C caller of the public ABI: compiles against include/slmopt.h as strict
 * C11 (the header a Go, Rust or Java binding would be generated from) and
 * links the library, then exercises the entry points that need no GPU. */
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "slmopt.h"

#define CHECK(c)                                                    \
  do {                                                              \
    if (!(c)) {                                                     \
      printf("FAIL %s:%d: %s\n", __FILE__, __LINE__, #c);           \
      return 1;                                                     \
    }                                                               \
  } while (0)

int main(void) {
  CHECK(slm_abi_version() == SLMOPT_ABI_VERSION);
  CHECK(strcmp(slm_status_code_string(SLM_OK), "OK") == 0);
  CHECK(strcmp(slm_status_code_string(SLM_ERR_MODEL_GRADIENT_NONFINITE),
               "MODEL_GRADIENT_NONFINITE") == 0);
  CHECK(slm_status_category(SLM_OK) == 0);
  CHECK(slm_status_category(SLM_ERR_MODEL_GRADIENT_NONFINITE) == 5); /* Gate */
  CHECK(slm_status_category(SLM_ERR_P12_SCHEDULER_STATE_MISMATCH) == 3); /* Integrity */
  CHECK(slm_status_category(SLM_ERR_INVALID_ARGUMENT) == 2); /* Usage */

  /* The reference's schedule, bit for bit: warmup ends at its peak, 3e-4. */
  float lr = 0.0f;
  CHECK(slm_canonical_learning_rate(0, &lr) != SLM_OK); /* updates count from 1 */
  CHECK(slm_canonical_learning_rate(1, &lr) == SLM_OK && lr > 0.0f);

  /* Sizes and argument checks answered before any device work. */
  CHECK(slm_gradient_clip_workspace_bytes(0) == 0);
  CHECK(slm_gradient_clip_workspace_bytes(135285504ull) == 478944ull);
  CHECK(slm_gradient_clip_scale_ws(NULL, 10, NULL, 0, NULL, NULL) == SLM_ERR_INVALID_ARGUMENT);
  CHECK(strlen(slm_last_error_message()) > 0);
  CHECK(slm_opt_create(NULL, 0, 0, NULL) == SLM_ERR_INVALID_ARGUMENT);
  CHECK(slm_opt_destroy(NULL) == SLM_OK);
  printf("ok\n");
  return 0;
}
