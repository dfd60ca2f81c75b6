/* The C ABI used from plain C99, as a Rust `extern "C"` block or cgo would
 * bind it: links libmmn_optim_cuda.so and runs the entry points that need no
 * GPU (defaults, version, routing, the sharding plan, argument checks). */
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "mmn_optim.h"

static int failures = 0;

#define CHECK(cond)                                              \
  do {                                                           \
    if (!(cond)) {                                               \
      fprintf(stderr, "%s:%d: check failed: %s\n", __FILE__, __LINE__, #cond); \
      ++failures;                                                \
    }                                                            \
  } while (0)

int main(void) {
  CHECK(mmn_abi_version() == MMN_OPTIM_ABI_VERSION);

  /* crates/mmn-optim/src/lib.rs:13-21 and :71-80 defaults */
  mmn_adamw_config a = mmn_adamw_config_default();
  CHECK(a.lr == 3e-4f && a.beta1 == 0.9f && a.beta2 == 0.95f && a.eps == 1e-8f &&
        a.weight_decay == 0.01f);
  mmn_muon_config m = mmn_muon_config_default();
  CHECK(m.lr == 0.02f && m.momentum == 0.95f && m.nesterov == 1 && m.ns_steps == 5);
  mmn_optim_config c = mmn_optim_config_default();
  CHECK(c.use_hybrid == 1 && c.world_size == 1 && c.rank == 0 && c.ns_mode == MMN_NS_REFERENCE);

  /* lib.rs:196-209: 2-D with both dims > 1 -> Muon, else AdamW */
  const int64_t mat[2] = {64, 256}, row[2] = {1, 64}, vec[1] = {64};
  CHECK(mmn_hybrid_classify_param(mat, 2) == MMN_ROUTE_MUON);
  CHECK(mmn_hybrid_classify_param(row, 2) == MMN_ROUTE_ADAMW);
  CHECK(mmn_hybrid_classify_param(vec, 1) == MMN_ROUTE_ADAMW);

  /* the plan of two equal matrices and one vector over two ranks: one matrix
   * per rank, the vector's AdamW range split between them */
  const int64_t shapes[5] = {128, 128, 128, 128, 1000};
  const int ndims[3] = {2, 2, 1};
  const int routes[3] = {MMN_ROUTE_AUTO, MMN_ROUTE_AUTO, MMN_ROUTE_AUTO};
  int owner[3] = {-9, -9, -9};
  int64_t offset[3] = {-1, -1, -1}, adamw_region = 0, muon_region = 0;
  CHECK(mmn_optim_plan(shapes, ndims, routes, 3, 1, 5, 2, owner, offset, &adamw_region,
                       &muon_region) == MMN_OK);
  CHECK(owner[0] >= 0 && owner[1] >= 0 && owner[0] != owner[1] && owner[2] == -1);
  CHECK(muon_region >= 128 * 128 && adamw_region * 2 >= 1000);

  /* errors come back as codes with a message, before any device is touched */
  mmn_optim_t *h = NULL;
  c.world_size = 0;
  CHECK(mmn_optim_create(&c, 0, NULL, &h) == MMN_E_INVALID && h == NULL);
  CHECK(strlen(mmn_last_error()) > 0);
  CHECK(mmn_optim_step(NULL, 1.0f) == MMN_E_INVALID);
  CHECK(mmn_optim_destroy(NULL) == MMN_OK);
  const void *srcs[1] = {NULL};
  CHECK(mmn_grad_reduce(srcs, 1, (void *)srcs, 16, MMN_DTYPE_F32, NULL, 0, NULL) ==
        MMN_E_INVALID);
  int *flags[1] = {NULL};
  CHECK(mmn_grad_nonfinite_scan(NULL, 16, MMN_DTYPE_F32, flags, 1, 0, NULL) == MMN_E_INVALID);

  if (failures) {
    fprintf(stderr, "%d check(s) failed\n", failures);
    return 1;
  }
  printf("c abi ok\n");
  return 0;
}
