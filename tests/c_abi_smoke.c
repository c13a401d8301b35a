/* The C ABI seen from C: compiled against include/hive_b200.h and linked to
 * libhive_b200.so by tests/test_c_abi.py. Makes no GPU call that could succeed on a
 * machine without a GPU: the version, the kernel list, argument errors with their
 * messages, and hv_init's status. Prints one "key=value" line per check. */
#include <stdio.h>
#include <string.h>

#include "hive_b200.h"

int main(void) {
  char buf[1024];
  printf("version=%d\n", hv_version());
  printf("abi_macro=%d\n", HV_ABI_VERSION);
  if (hv_kernel_list(buf, sizeof buf) != HV_OK) return 2;
  printf("has_k_step=%d\n", strstr(buf, "k_step") != NULL);
  int rc = hv_a4gv(NULL, NULL, NULL, NULL, NULL, 8, 16, NULL);
  hv_last_error(buf, sizeof buf);
  printf("a4gv_null_rc=%d\n", rc);
  printf("a4gv_null_msg=%s\n", buf);
  rc = hv_wait_probe(NULL, 1, 1, 1000, NULL, NULL);
  printf("wait_probe_null_rc=%d\n", rc);
  rc = hv_argmax_key_final(NULL, 0, NULL, NULL, NULL, NULL, NULL);
  printf("argmax_key_final_null_rc=%d\n", rc);
  size_t nib = 0, sc = 0;
  rc = hv_w4_prepacked_size(24, 4096, 12, &nib, &sc);
  printf("prepacked_rc=%d nib=%zu sc=%zu\n", rc, nib, sc);
  rc = hv_init();
  hv_last_error(buf, sizeof buf);
  printf("init_rc=%d\n", rc);
  printf("init_msg_nonempty=%d\n", rc == HV_OK || buf[0] != 0);
  return 0;
}
