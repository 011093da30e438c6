/* A plain C caller of the library (C99, no C++): the header compiles as C
 * and host-only entry points work without a GPU. Built and run by
 * tests/test_abi.py; exits non-zero on the first wrong answer. */
#include <stdio.h>
#include <string.h>

#include "inferox.h"

int main(void) {
  ifx_load_opts o;
  ifx_load_opts_default(&o);
  if (o.tp_size != 1 || o.kquant_layout != IFX_KQUANT_REFERENCE || o.tp_timeout_ms != 0) return 1;
  if (strcmp(ifx_status_name(IFX_ERR_JSON), "Json") != 0) return 2;
  if (ifx_version() <= 0) return 3;
  const char *json =
      "{\"model\": {\"type\": \"BPE\", \"vocab\": {\"a\": 1, \"b\": 2, \"ab\": 3},"
      " \"merges\": [\"a b\"]}}";
  ifx_tokenizer *t = NULL;
  if (ifx_tokenizer_load_json(json, strlen(json), &t) != IFX_OK) return 4;
  uint32_t ids[8];
  size_t n = 0;
  if (ifx_tokenizer_encode(t, "abab", 4, ids, 8, &n) != IFX_OK || n != 2 || ids[0] != 3 ||
      ids[1] != 3)
    return 5;
  char text[16];
  size_t len = 0;
  if (ifx_tokenizer_decode(t, ids, n, text, sizeof text, &len) != IFX_OK || len != 4 ||
      memcmp(text, "abab", 4) != 0)
    return 6;
  ifx_tokenizer_free(t);
  unsigned char blk[34] = {0}, out[34];
  int ty = -1, sgn = -1;
  if (ifx_kquant_from_ggml(8, blk, sizeof blk, out, &ty, &sgn) != IFX_OK || ty != IFX_TYPE_Q8_0 ||
      sgn != 0)
    return 7;
  puts("c caller ok");
  return 0;
}
