/*
 * A plain C99 consumer of libsemantica_b200.so: the calls a Go host makes
 * through cgo, made from C with nothing but include/semantica_b200.h.
 *
 *   abi_consumer link
 *       calls sem_device_count and sem_last_error only (no GPU needed);
 *   abi_consumer run <model.gguf> <ids.bin> <out.bin>
 *       ids.bin: int32 n_seqs, int32 offsets[n_seqs + 1], int32 ids[...],
 *       int32 dims[n_seqs]; embeds them with sem_embed and writes the packed
 *       vectors (float32) to out.bin, then exercises the request pipeline,
 *       an error string, a small int8 index (search, serialise, deserialise)
 *       and prints one "ok" line per check.
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "semantica_b200.h"

#define CHECK(call)                                                                 \
  do {                                                                              \
    int rc_ = (call);                                                               \
    if (rc_ != SEM_OK) {                                                            \
      fprintf(stderr, "%s failed (%d): %s\n", #call, rc_, sem_last_error());        \
      return 1;                                                                     \
    }                                                                               \
  } while (0)

static int32_t *read_all(const char *path, long *n_words) {
  FILE *f = fopen(path, "rb");
  if (!f) return NULL;
  fseek(f, 0, SEEK_END);
  long bytes = ftell(f);
  fseek(f, 0, SEEK_SET);
  int32_t *buf = (int32_t *)malloc((size_t)bytes);
  if (buf && fread(buf, 1, (size_t)bytes, f) != (size_t)bytes) {
    free(buf);
    buf = NULL;
  }
  fclose(f);
  *n_words = bytes / 4;
  return buf;
}

static int link_mode(void) {
  int n = -1;
  int rc = sem_device_count(&n);
  printf("device_count rc=%d n=%d last_error=%s\n", rc, n, sem_last_error());
  return 0;
}

/* deterministic pseudo-random floats in [-1, 1) */
static float lcg(uint32_t *s) {
  *s = *s * 1664525u + 1013904223u;
  return (float)((*s >> 8) & 0xffffff) / 8388608.0f - 1.0f;
}

static int run_mode(const char *model_path, const char *ids_path, const char *out_path) {
  long nw = 0;
  int32_t *in = read_all(ids_path, &nw);
  if (!in || nw < 2) {
    fprintf(stderr, "cannot read %s\n", ids_path);
    return 1;
  }
  const int32_t n = in[0];
  const int32_t *offsets = in + 1;
  const int32_t *ids = offsets + n + 1;
  const int32_t *dims = ids + offsets[n];
  long floats = 0;
  for (int s = 0; s < n; ++s) floats += dims[s];

  sem_context *ctx = NULL;
  sem_model *model = NULL;
  CHECK(sem_context_create(0, &ctx));
  CHECK(sem_model_load_gguf(ctx, model_path, &model));
  sem_model_config cfg;
  CHECK(sem_model_config_get(model, &cfg));

  float *out = (float *)malloc((size_t)floats * sizeof(float));
  CHECK(sem_embed(model, ids, offsets, n, dims, out));
  FILE *f = fopen(out_path, "wb");
  if (!f || fwrite(out, sizeof(float), (size_t)floats, f) != (size_t)floats) return 1;
  fclose(f);
  printf("ok embed %d sequences, %ld floats\n", n, floats);

  /* the request pipeline gives the same vectors */
  float *out2 = (float *)malloc((size_t)floats * sizeof(float));
  uint64_t t0 = 0, t1 = 0;
  CHECK(sem_embed_submit(model, ids, offsets, n, dims, &t0));
  CHECK(sem_embed_submit(model, ids, offsets, n, dims, &t1));
  CHECK(sem_embed_wait(model, t0, out2));
  if (memcmp(out, out2, (size_t)floats * sizeof(float)) != 0) return 2;
  CHECK(sem_embed_wait(model, t1, out2));
  if (memcmp(out, out2, (size_t)floats * sizeof(float)) != 0) return 2;
  printf("ok pipeline\n");

  /* the reference's error string */
  {
    const int32_t bad_ids[2] = {2, cfg.vocab_size};
    const int32_t bad_off[2] = {0, 2};
    const int32_t bad_dim[1] = {cfg.embed_dim};
    float v[1024];
    int rc = sem_embed(model, bad_ids, bad_off, 1, bad_dim, v);
    char want[64];
    snprintf(want, sizeof want, "token ID out of range: %d", cfg.vocab_size);
    if (rc != SEM_EINVAL || strcmp(sem_last_error(), want) != 0) return 3;
    printf("ok error string\n");
  }

  /* a small int8 index: build, exact search, BRUT round trip */
  {
    enum { COUNT = 2000, DIM = 128, NQ = 4, K = 5 };
    float *vecs = (float *)malloc(sizeof(float) * COUNT * DIM);
    int32_t *vid = (int32_t *)malloc(sizeof(int32_t) * COUNT);
    uint32_t seed = 12345u;
    for (int i = 0; i < COUNT * DIM; ++i) vecs[i] = lcg(&seed);
    for (int i = 0; i < COUNT; ++i) vid[i] = 1000 + i;
    sem_index *idx = NULL, *idx2 = NULL;
    CHECK(sem_index_build(ctx, DIM, 1, vecs, vid, COUNT, &idx));
    /* queries: the first NQ stored vectors, so each finds itself first */
    int32_t got[NQ * K], got2[NQ * K];
    float dist[NQ * K], dist2[NQ * K];
    CHECK(sem_index_search(idx, vecs, NQ, DIM, K, SEM_SEARCH_EXACT, 1, got, dist, NULL));
    for (int q = 0; q < NQ; ++q)
      if (got[q * K] != 1000 + q) return 4;
    size_t need = 0, written = 0;
    CHECK(sem_index_serialize(idx, NULL, 0, &need));
    void *bytes = malloc(need);
    CHECK(sem_index_serialize(idx, bytes, need, &written));
    if (written != need || memcmp(bytes, "BRUT", 4) != 0) return 5;
    CHECK(sem_index_deserialize(ctx, bytes, written, &idx2));
    CHECK(sem_index_search(idx2, vecs, NQ, DIM, K, SEM_SEARCH_EXACT, 1, got2, dist2, NULL));
    if (memcmp(got, got2, sizeof got) != 0 || memcmp(dist, dist2, sizeof dist) != 0) return 6;
    printf("ok index (%zu BRUT bytes)\n", written);
    sem_index_free(idx2);
    sem_index_free(idx);
    free(bytes);
    free(vid);
    free(vecs);
  }

  CHECK(sem_model_free(model));
  CHECK(sem_context_destroy(ctx));
  free(out2);
  free(out);
  free(in);
  printf("ok done\n");
  return 0;
}

int main(int argc, char **argv) {
  if (argc >= 2 && strcmp(argv[1], "link") == 0) return link_mode();
  if (argc == 5 && strcmp(argv[1], "run") == 0) return run_mode(argv[2], argv[3], argv[4]);
  fprintf(stderr, "usage: abi_consumer link | run <model.gguf> <ids.bin> <out.bin>\n");
  return 64;
}
