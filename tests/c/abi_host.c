/* A plain C (C99) caller of libnvkv.so's host entry points: the header must
 * compile as C and the ABI must work without C++ or Python.  Exercises the
 * block manager (admission with a prefix-cache hit, decode growth through
 * the batched append) and the step-metadata builder; prints one line of
 * results that tests/test_c_abi.py checks. */
#include <stdio.h>
#include <stdlib.h>

#include "nvkv.h"

#define CHECK(x)                                                         \
  do {                                                                   \
    int rc_ = (x);                                                       \
    if (rc_ != NVKV_OK) {                                                \
      fprintf(stderr, "%s failed: %d %s\n", #x, rc_, nvkv_last_error()); \
      return 1;                                                          \
    }                                                                    \
  } while (0)

int main(void) {
  enum { BS = 4, NB = 16, LEN = 10, CAP = 32 };
  uint32_t toks[2][CAP];
  uint32_t tables[2][CAP];
  nvkv_block_seq seqs[2];
  nvkv_block_manager_t bm = NULL;
  int64_t used = 0, freeb = 0, fresh = 0, done = 0, nfree = 0;
  int64_t one[2] = {1, 1};
  int s, i;
  CHECK(nvkv_block_manager_create(NB, BS, &bm));
  for (s = 0; s < 2; ++s) {
    for (i = 0; i < LEN; ++i) toks[s][i] = (uint32_t)(i < 8 ? 100 + i : 200 + 10 * s + i);
    seqs[s].token_ids = toks[s];
    seqs[s].num_tokens = LEN;
    seqs[s].num_cached_tokens = 0;
    seqs[s].block_table = tables[s];
    seqs[s].block_table_len = 0;
    seqs[s].block_table_capacity = CAP;
    CHECK(nvkv_block_manager_get_token_layout(bm, &seqs[s], &used, &freeb, &fresh));
    seqs[s].num_new_tokens = fresh;
    CHECK(nvkv_block_manager_allocate(bm, &seqs[s]));
    seqs[s].num_cached_tokens += seqs[s].num_new_tokens;
    seqs[s].num_new_tokens = 0;
  }
  /* the second sequence shares the first two pages (8 common tokens) */
  printf("cached=%lld shared=%d ", (long long)used,
         tables[0][0] == tables[1][0] && tables[0][1] == tables[1][1]);
  for (s = 0; s < 2; ++s) {
    toks[s][seqs[s].num_tokens] = 7;
    seqs[s].num_tokens += 1;
  }
  CHECK(nvkv_block_manager_append_batch(bm, seqs, 2, one, &done));
  {
    nvkv_step_sizes z;
    int64_t ids[8], pos[8], slots[8], ctx[2], logits[2];
    uint32_t cuq[3], cuk[3], bt[2 * CAP];
    CHECK(nvkv_prepare_step(seqs, 2, BS, NULL, NULL, NULL, NULL, NULL, NULL, NULL, NULL, 0, 0,
                            0, &z));
    CHECK(nvkv_prepare_step(seqs, 2, BS, ids, pos, cuq, cuk, slots, ctx, logits, bt, 8, 8,
                            2 * CAP, &z));
    CHECK(nvkv_block_manager_num_free(bm, &nfree));
    printf("done=%lld tokens=%lld slots=%lld cuk=%u,%u,%u pos=%lld,%lld slot0=%lld free=%lld\n",
           (long long)done, (long long)z.num_tokens, (long long)z.num_slots, cuk[0], cuk[1],
           cuk[2], (long long)pos[0], (long long)pos[1], (long long)slots[0], (long long)nfree);
  }
  CHECK(nvkv_block_manager_destroy(bm));
  return 0;
}
