/* The C ABI from plain C99: include/scunet_b200.h compiled as C, linked against the
 * built library, and called the way a non-C++ host (a Rust `impl Backend` through
 * its FFI, a Go program through cgo) calls it. It builds the full tensor table of
 * scunet-rs src/weights.rs:207-263 by name - the walk a Rust binding does over
 * `Weights::t(name)` - with zero-filled data, then:
 *   - checks the host-side refusals (missing tensor, bad architecture, NULL ctx);
 *   - checks scb_need_bytes (pure arithmetic);
 *   - calls scb_create: without a usable B200 it must fail with SCB_ECUDA and a
 *     message (no CPU fallback); with one it must succeed, report its footprint and
 *     memory, and be destroyed.
 * Exit status 0 = every check passed. Built and run by tests/test_native_cpu.py. */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "scunet_b200.h"

#define MAXT 640
static scb_tensor tab[MAXT];
static char names[MAXT][96];
static int nt = 0;
static float* zeros = NULL;
static int failures = 0;

#define CHECK(cond)                                                   \
  do {                                                                \
    if (!(cond)) {                                                    \
      fprintf(stderr, "FAILED line %d: %s\n", __LINE__, #cond);       \
      ++failures;                                                     \
    }                                                                 \
  } while (0)

static void add(const char* name, int ndim, int64_t d0, int64_t d1, int64_t d2, int64_t d3) {
  scb_tensor* t = &tab[nt];
  snprintf(names[nt], sizeof names[nt], "%s", name);
  t->name = names[nt];
  t->data = zeros;
  t->ndim = ndim;
  t->shape[0] = d0;
  t->shape[1] = d1;
  t->shape[2] = d2;
  t->shape[3] = d3;
  ++nt;
}

/* One ConvTransBlock of a plane with c channels (c/2 conv, c/2 trans). */
static void block(const char* pre, int c) {
  const int t = c / 2, heads = t / 32;
  char n[96];
#define NM(suffix) (snprintf(n, sizeof n, "%s.%s", pre, suffix), n)
  add(NM("conv1_1.weight"), 4, c, c, 1, 1);
  add(NM("conv1_1.bias"), 1, c, 0, 0, 0);
  add(NM("conv1_2.weight"), 4, c, c, 1, 1);
  add(NM("conv1_2.bias"), 1, c, 0, 0, 0);
  add(NM("conv_block.0.weight"), 4, t, t, 3, 3);
  add(NM("conv_block.2.weight"), 4, t, t, 3, 3);
  add(NM("trans_block.ln1.weight"), 1, t, 0, 0, 0);
  add(NM("trans_block.ln1.bias"), 1, t, 0, 0, 0);
  add(NM("trans_block.ln2.weight"), 1, t, 0, 0, 0);
  add(NM("trans_block.ln2.bias"), 1, t, 0, 0, 0);
  add(NM("trans_block.msa.embedding_layer.weight"), 2, 3 * t, t, 0, 0);
  add(NM("trans_block.msa.embedding_layer.bias"), 1, 3 * t, 0, 0, 0);
  add(NM("trans_block.msa.linear.weight"), 2, t, t, 0, 0);
  add(NM("trans_block.msa.linear.bias"), 1, t, 0, 0, 0);
  add(NM("trans_block.msa.relative_position_params"), 3, heads, 15, 15, 0);
  add(NM("trans_block.mlp.0.weight"), 2, 4 * t, t, 0, 0);
  add(NM("trans_block.mlp.0.bias"), 1, 4 * t, 0, 0, 0);
  add(NM("trans_block.mlp.2.weight"), 2, t, 4 * t, 0, 0);
  add(NM("trans_block.mlp.2.bias"), 1, t, 0, 0, 0);
#undef NM
}

static void table(int in_nc) {
  static const char* stage[7] = {"down1", "down2", "down3", "body", "up3", "up2", "up1"};
  static const int level[7] = {0, 1, 2, 3, 2, 1, 0};
  char n[96];
  int s, i;
  nt = 0;
  add("m_head.0.weight", 4, 64, in_nc, 3, 3);
  add("m_tail.0.weight", 4, in_nc, 64, 3, 3);
  for (s = 0; s < 7; ++s) {
    const int c = 64 << level[s], first = s >= 4 ? 1 : 0;
    for (i = 0; i < 4; ++i) {
      snprintf(n, sizeof n, "m_%s.%d", stage[s], first + i);
      block(n, c);
    }
    if (s < 3) {
      snprintf(n, sizeof n, "m_%s.4.weight", stage[s]);
      add(n, 4, 2 * c, c, 2, 2);
    }
    if (s >= 4) {
      snprintf(n, sizeof n, "m_%s.0.weight", stage[s]);
      add(n, 4, 2 * c, c, 2, 2);
    }
  }
}

int main(void) {
  const int config[7] = {4, 4, 4, 4, 4, 4, 4};
  scb_ctx* ctx = NULL;
  size_t bytes = 0;
  int rc;
  zeros = (float*)calloc(1 << 20, sizeof(float)); /* >= the largest tensor (589,824 values) */
  if (!zeros) return 2;
  table(3);
  CHECK(nt == 2 + 28 * 19 + 3 + 3);

  /* pure arithmetic: the memguard figure for one padded 1920x1088 frame */
  CHECK(scb_need_bytes(1, 3, 1088, 1920, &bytes) == SCB_OK);
  CHECK(bytes > (size_t)1000 * 1088 * 1920 && bytes < (size_t)1400 * 1088 * 1920);
  CHECK(scb_need_bytes(1, 3, 1080, 1920, &bytes) == SCB_EINVAL); /* not padded */

  /* host-side refusals, before any device work */
  rc = scb_create(tab, nt - 1, 3, 64, 32, 8, config, 0, &ctx); /* the last tensor is missing */
  CHECK(rc == SCB_ENOWEIGHT && ctx == NULL && strstr(scb_last_error(NULL), "m_up1.0.weight") != NULL);
  rc = scb_create(tab, nt, 2, 64, 32, 8, config, 0, &ctx);
  CHECK(rc == SCB_EINVAL && strstr(scb_last_error(NULL), "in_nc") != NULL);
  CHECK(scb_forward_dev(NULL, NULL, SCB_U8, 1, 3, 64, 64, NULL, SCB_F32, NULL) == SCB_EINVAL);
  CHECK(scb_mem_report(NULL, NULL, NULL, NULL) == SCB_EINVAL);
  scb_destroy(NULL);
  scb_release_scratch(NULL);

  /* the full table: a B200 or a loud failure */
  rc = scb_create(tab, nt, 3, 64, 32, 8, config, 0, &ctx);
  if (rc == SCB_OK) {
    size_t wb = 0, sb = 0, hw = 0, live = 0, fixed = 0;
    scb_footprint(ctx, &wb, &sb);
    CHECK(wb > 30u << 20 && sb == 0);
    CHECK(scb_mem_report(ctx, &hw, &live, &fixed) == SCB_OK && hw >= wb && live == wb && fixed == 14u << 20);
    scb_destroy(ctx);
    printf("abi ok (device present)\n");
  } else {
    CHECK(rc == SCB_ECUDA && ctx == NULL && strlen(scb_last_error(NULL)) > 0);
    printf("abi ok (no device: %s)\n", scb_last_error(NULL));
  }
  free(zeros);
  return failures ? 1 : 0;
}
