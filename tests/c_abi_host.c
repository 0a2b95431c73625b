/* A plain C host of libattention_decode_b200 (built by tests/test_cabi.py):
 * the header must compile as C and every call below is answered on the host,
 * without a GPU.  Prints one line per check; exits non-zero on a mismatch. */
#include <stdio.h>
#include <string.h>

#include "attention_decode_b200.h"

static int failures = 0;

static void expect(const char* what, int got, int want) {
  printf("%s: status %d (%s)\n", what, got, got == ADB_OK ? "ok" : adb_last_error());
  if (got != want) {
    printf("  expected %d\n", want);
    ++failures;
  }
}

int main(void) {
  size_t bytes = 0;
  printf("version: %s\n", adb_version());
  if (strstr(adb_version(), "sm_100a") == NULL) ++failures;
  expect("decode with null pointers",
         adb_decode(NULL, NULL, NULL, NULL, NULL, 1, 32, 8, 129, 128, NULL, 0, 0, 0, NULL),
         ADB_ERR_INVALID_ARGUMENT);
  expect("group of 16", adb_decode_workspace_size(1, 32, 2, 129, 128, 0, 0, &bytes, NULL),
         ADB_ERR_UNSUPPORTED);
  expect("exchange size, 8 ranks", adb_exchange_size(64, 128, 8, &bytes), ADB_OK);
  if (bytes != 256 + 2 * 8 * 64 * 128 * 4 + 2 * 8 * 64 * 2 * 4) ++failures;
  expect("paged, page size 12",
         adb_decode_paged(NULL, NULL, NULL, (const int32_t*)8, 4, (const int32_t*)8, NULL, 2, 32, 8,
                          128, 16, 12, 4, ADB_PAGED_HND, NULL, 0, 0, 0, NULL),
         ADB_ERR_UNSUPPORTED);
  expect("fp8, zero scale",
         adb_decode_fp8(NULL, NULL, NULL, NULL, NULL, 1, 32, 8, 129, 128, 0.0f, 1.0f, NULL, 0, 0, 0, NULL),
         ADB_ERR_INVALID_ARGUMENT);
  printf("%s\n", failures ? "FAILED" : "all host checks passed");
  return failures ? 1 : 0;
}
