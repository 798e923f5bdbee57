// Model loading and the batched forward pass (the host side of
// internal/runtime: LoadModel model.go:233-315, ForwardWithDim model.go:661-666,
// forwardINT8WithDim model_int8.go:148-256).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "gguf.h"
#include "internal.h"

namespace sem {

namespace {
thread_local std::string g_error;
}

int set_error(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_error = buf;
  return code;
}

const char* last_error() { return g_error.c_str(); }

struct LayerW {
  Q8Proj qkv, o, gu, down;  // gu = gate rows then up rows
  float *attn_norm, *q_norm, *k_norm, *post_attn, *ffn_norm, *post_ffw;
};

}  // namespace sem

struct sem_model {
  sem_context* ctx = nullptr;
  sem_model_config cfg{};
  sem::DevBuf arena;  // all weights
  int8_t* emb = nullptr;
  float* emb_s = nullptr;
  float* out_norm = nullptr;
  float* rope_cos = nullptr;
  float* rope_sin = nullptr;
  std::vector<sem::LayerW> layers;
  // forward workspaces (grow only)
  sem::DevBuf hid, big, att, codes, halves, inv_rms, meta, absmax, ids, ids_in, out, errflag;
  int64_t ws_T = -1;
  // cached metadata of the last batch shape
  std::vector<int32_t> last_offsets, last_dims;
  int32_t n_tiles = 0;
  int32_t n_tiles_long = 0;  // attention tiles of the long sequences (first in the tile list)
  int32_t n_ptiles = 0, n_ptiles_long = 0;  // 256-row tiles of the SM-pair attention (all, long sequences')
  int32_t short_max_len = 0; // longest sequence under kSplitMinLen tokens
  int64_t t_long = 0;     // packed rows of the long sequences (first in the packed order)
  bool permuted = false;  // packed order differs from the caller's
  // optional per-launch timing
  bool prof = false;
  std::vector<cudaEvent_t> prof_events;  // pairs (before, after)
  std::vector<int> prof_stage;           // stage of each pair
  size_t prof_used = 0;                  // events recorded since the last read
  double prof_ms[16] = {0};
  int32_t prof_n[16] = {0};
  // CUDA graphs of the forwards of recent small batch shapes (sem_embed,
  // sem_embed_submit), each with the buffers, projection path, stream and
  // shape it was captured for; the least recently replayed goes first
  struct Graph {
    std::vector<const void*> key;
    std::vector<int32_t> shape;  // offsets[0..B] then dims[0..B)
    cudaGraphExec_t exec = nullptr;
    uint64_t used = 0;
  };
  std::vector<Graph> graphs;
  uint64_t graph_tick = 0;
  bool graphs_off = false;  // a capture failed here: forwards run without a graph
  // sem_embed_submit / sem_embed_wait: two request slots, each with pinned
  // staging for its ids, metadata, outputs and error words, so the host
  // prepares one request while the device runs the other
  struct Slot {
    sem::HostBuf ids, meta, out, flags;
    cudaEvent_t done = nullptr;
    uint64_t ticket = 0;
    bool busy = false;
    int64_t out_floats = 0;
  };
  Slot slots[2];
  uint64_t next_ticket = 1;
  // model-faithful mode (sem_model_set_faithful): sliding-window layers, their
  // RoPE tables, the dense 2/3 head (weights loaded when the file has them)
  sem_faithful_config faithful{};
  uint32_t faithful_gen = 0;  // changes with the mode: cached graphs are re-captured
  sem::DevBuf rope_swa;       // cos then sin tables of the sliding layers' base
  sem::DevBuf dense_buf;      // dense_2 and dense_3 in every projection layout
  sem::Q8Proj dense2{}, dense3{};
  int32_t dense_mid = 0;      // dense_2 output width
  sem::DevBuf head_y1, head_codes, head_absmax;
};


namespace sem {
namespace {

constexpr uint32_t kF32 = 0, kQ8 = 8;

const sem_tensor_view* find_view(const sem_tensor_view* v, int n, const std::string& name) {
  for (int i = 0; i < n; ++i)
    if (v[i].name && name == v[i].name) return &v[i];
  return nullptr;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Raw upload of one Q8_0 tensor into the staging buffer, then the repack kernel.
int upload_q8(sem_context* ctx, DevBuf& staging, const sem_tensor_view* t, int64_t rows, int cols, int8_t* codes,
              float* scales, int64_t row_off, int interleave, int part, bool gguf_dec) {
  uint64_t need = (uint64_t)rows * (cols / 32) * 34;
  if (t->nbytes < need) return set_error(SEM_EFORMAT, "tensor %s: %llu bytes, need %llu", t->name,
                                         (unsigned long long)t->nbytes, (unsigned long long)need);
  SEM_CUDA(staging.ensure(need));
  SEM_CUDA(cudaMemcpyAsync(staging.p, t->data, need, cudaMemcpyHostToDevice, ctx->stream));
  SEM_CUDA(launch_repack_q8_0(staging.as<uint8_t>(), rows, cols, codes, scales, row_off, interleave, part, gguf_dec,
                              ctx->stream));
  // the staging buffer is reused by the next tensor: finish this one first
  SEM_CUDA(cudaStreamSynchronize(ctx->stream));
  return SEM_OK;
}

// Same for a projection weight, every layout of the GEMMs at rows
// [row_off, row_off + rows): fp16 codes with fp32 block scales, the split fp16
// planes with their row scales, and the lane-major int8 plane.
int upload_q8_proj(sem_context* ctx, DevBuf& staging, const sem_tensor_view* t, int64_t rows, int cols,
                   const Q8Proj& w, int64_t row_off) {
  uint64_t need = (uint64_t)rows * (cols / 32) * 34;
  if (t->nbytes < need) return set_error(SEM_EFORMAT, "tensor %s: %llu bytes, need %llu", t->name,
                                         (unsigned long long)t->nbytes, (unsigned long long)need);
  SEM_CUDA(staging.ensure(need));
  SEM_CUDA(cudaMemcpyAsync(staging.p, t->data, need, cudaMemcpyHostToDevice, ctx->stream));
  SEM_CUDA(launch_repack_q8_0_f16(staging.as<uint8_t>(), rows, cols, const_cast<__half*>(w.codes),
                                  const_cast<float*>(w.scales), row_off, ctx->stream));
  SEM_CUDA(launch_repack_q8_0_split(staging.as<uint8_t>(), rows, cols, const_cast<__half*>(w.hi),
                                    const_cast<__half*>(w.lo), const_cast<float*>(w.row_scale), row_off, ctx->stream));
  SEM_CUDA(launch_repack_q8_0_lanes(staging.as<uint8_t>(), rows, cols, const_cast<int8_t*>(w.lanes), row_off,
                                    ctx->stream));
  SEM_CUDA(cudaStreamSynchronize(ctx->stream));
  return SEM_OK;
}

int check_q8(const sem_tensor_view* t, const char* name, uint64_t k, uint64_t n) {
  if (!t) return set_error(SEM_ENOTFOUND, "tensor not found: %s", name);
  if (t->dtype != kQ8) return set_error(SEM_EFORMAT, "expected Q8_0, got dtype %u for %s", t->dtype, name);
  if (t->n_dims < 2 || t->dims[0] != k || t->dims[1] != n)
    return set_error(SEM_EFORMAT, "tensor %s: shape {%llu,%llu}, want {%llu,%llu}", name,
                     (unsigned long long)t->dims[0], (unsigned long long)(t->n_dims > 1 ? t->dims[1] : 0),
                     (unsigned long long)k, (unsigned long long)n);
  return SEM_OK;
}

}  // namespace

// ---------------------------------------------------------------------------
// Model load
// ---------------------------------------------------------------------------
int model_load(sem_context* ctx, const sem_model_config* cfg_in, const sem_tensor_view* tv, int nt, sem_model** out) {
  if (!ctx || !cfg_in || !tv || !out) return set_error(SEM_EINVAL, "null argument");
  const sem_model_config c = *cfg_in;
  const int H = c.embed_dim, F = c.interm_dim, L = c.num_layers, nh = c.num_heads, hd = c.head_dim;
  // shapes the sm_100a kernels are built for (EmbeddingGemma-300M and its variants)
  if (hd != 256 || c.num_kv_heads != 1 || nh < 1 || nh > 3 || H != nh * hd || H % 128 || F % 128 || L < 1 ||
      c.vocab_size < 1 || c.max_seq_len < 1)
    return set_error(SEM_EINVAL,
                     "unsupported model shape: embed_dim=%d heads=%d kv_heads=%d head_dim=%d ffn=%d (need head_dim 256, "
                     "1 KV head, <=3 query heads, embed_dim%%128==0, ffn%%128==0)",
                     H, nh, c.num_kv_heads, hd, F);
  DeviceGuard dg(ctx->device);
  std::lock_guard<std::mutex> lk(ctx->mu);
  std::unique_ptr<sem_model> m(new sem_model());
  m->ctx = ctx;
  m->cfg = c;
  const int qkvN = nh * hd + 2 * hd;
  const int64_t V = c.vocab_size;
  // ---- arena layout ----
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = align256(off + bytes);
    return o;
  };
  size_t o_emb = take((size_t)V * H), o_emb_s = take((size_t)V * (H / 32) * 4), o_onorm = take((size_t)H * 4);
  size_t o_cos = take((size_t)c.max_seq_len * (hd / 2) * 4), o_sin = take((size_t)c.max_seq_len * (hd / 2) * 4);
  // one projection [rows][k]: codes, block scales, hi, lo, row scales, int8 lanes
  struct POff { size_t codes, scales, hi, lo, rsc, lanes; };
  auto take_proj = [&](int64_t rows, int64_t k) {
    POff p;
    p.codes = take((size_t)rows * k * 2);
    p.scales = take((size_t)rows * (k / 32) * 4);
    p.hi = take((size_t)2 * rows * k * 2);  // hi plane, then the lo plane right after it
    p.lo = p.hi + (size_t)rows * k * 2;
    p.rsc = take((size_t)rows * 4);
    p.lanes = take((size_t)rows * k);
    return p;
  };
  struct LOff { POff qkv, o, gu, down; size_t an, qn, kn, pa, fn, pf; };
  std::vector<LOff> lo(L);
  for (int l = 0; l < L; ++l) {
    lo[l].qkv = take_proj(qkvN, H);
    lo[l].o = take_proj(H, H);
    lo[l].gu = take_proj(2 * F, H);
    lo[l].down = take_proj(H, F);
    lo[l].an = take(H * 4); lo[l].qn = take(hd * 4); lo[l].kn = take(hd * 4);
    lo[l].pa = take(H * 4); lo[l].fn = take(H * 4); lo[l].pf = take(H * 4);
  }
  cudaError_t e = m->arena.ensure(off);
  if (e != cudaSuccess) return set_error(SEM_ENOMEM, "device allocation of %zu bytes failed: %s", off, cudaGetErrorString(e));
  uint8_t* base = m->arena.as<uint8_t>();
  SEM_CUDA(cudaMemsetAsync(base, 0, off, ctx->stream));
  m->emb = reinterpret_cast<int8_t*>(base + o_emb);
  m->emb_s = reinterpret_cast<float*>(base + o_emb_s);
  m->rope_cos = reinterpret_cast<float*>(base + o_cos);
  m->rope_sin = reinterpret_cast<float*>(base + o_sin);
  DevBuf staging;
  int rc;
  // ---- token embedding (model.go:520-540), gguf f16 decoder ----
  const sem_tensor_view* te = find_view(tv, nt, "token_embd.weight");
  if (!te) te = find_view(tv, nt, "model.embed_tokens.weight");
  if (!te) return set_error(SEM_ENOTFOUND, "load weights: token embedding tensor not found");
  if (te->dtype != kQ8) return set_error(SEM_EFORMAT, "load weights: expected Q8_0 embeddings, got dtype %u", te->dtype);
  if (te->dims[0] != (uint64_t)H || te->dims[1] < (uint64_t)V)
    return set_error(SEM_EFORMAT, "token_embd.weight shape {%llu,%llu} does not cover vocab %lld x %d",
                     (unsigned long long)te->dims[0], (unsigned long long)te->dims[1], (long long)V, H);
  if ((rc = upload_q8(ctx, staging, te, V, H, m->emb, m->emb_s, 0, 0, 0, true))) return rc;
  // ---- F32 tensors ----
  auto up_f32 = [&](const char* name, size_t o, int n, bool required, float** dst) -> int {
    const sem_tensor_view* t = find_view(tv, nt, name);
    *dst = nullptr;
    if (!t) return required ? set_error(SEM_ENOTFOUND, "tensor not found: %s", name) : SEM_OK;
    if (t->dtype != kF32 || t->nbytes < (uint64_t)n * 4)
      return set_error(SEM_EFORMAT, "tensor %s: expected %d F32 values", name, n);
    *dst = reinterpret_cast<float*>(base + o);
    SEM_CUDA(cudaMemcpyAsync(*dst, t->data, (size_t)n * 4, cudaMemcpyHostToDevice, ctx->stream));
    return SEM_OK;
  };
  if ((rc = up_f32("output_norm.weight", o_onorm, H, false, &m->out_norm))) return rc;
  m->layers.resize(L);
  char nm[128];
  for (int l = 0; l < L; ++l) {
    LayerW& w = m->layers[l];
    auto P = [&](const char* s) { snprintf(nm, sizeof nm, "blk.%d.%s", l, s); return (const char*)nm; };
    if ((rc = up_f32(P("attn_norm.weight"), lo[l].an, H, true, &w.attn_norm))) return rc;
    if ((rc = up_f32(P("ffn_norm.weight"), lo[l].fn, H, true, &w.ffn_norm))) return rc;
    if ((rc = up_f32(P("attn_q_norm.weight"), lo[l].qn, hd, false, &w.q_norm))) return rc;
    if ((rc = up_f32(P("attn_k_norm.weight"), lo[l].kn, hd, false, &w.k_norm))) return rc;
    if ((rc = up_f32(P("post_attention_norm.weight"), lo[l].pa, H, false, &w.post_attn))) return rc;
    if ((rc = up_f32(P("post_ffw_norm.weight"), lo[l].pf, H, false, &w.post_ffw))) return rc;
    auto proj = [&](const POff& p) {
      return Q8Proj{reinterpret_cast<const __half*>(base + p.codes), reinterpret_cast<const float*>(base + p.scales),
                    reinterpret_cast<const __half*>(base + p.hi), reinterpret_cast<const __half*>(base + p.lo),
                    reinterpret_cast<const float*>(base + p.rsc), reinterpret_cast<const int8_t*>(base + p.lanes)};
    };
    w.qkv = proj(lo[l].qkv);
    w.o = proj(lo[l].o);
    w.gu = proj(lo[l].gu);
    w.down = proj(lo[l].down);
    // Q|K|V fused into one [qkvN][H] matrix, gate rows then up rows in [2F][H]
    struct { const char* n; uint64_t k, rows; const Q8Proj* w; int64_t roff; } q8[] = {
        {"attn_q.weight", (uint64_t)H, (uint64_t)nh * hd, &w.qkv, 0},
        {"attn_k.weight", (uint64_t)H, (uint64_t)hd, &w.qkv, (int64_t)nh * hd},
        {"attn_v.weight", (uint64_t)H, (uint64_t)hd, &w.qkv, (int64_t)nh * hd + hd},
        {"attn_output.weight", (uint64_t)H, (uint64_t)H, &w.o, 0},
        {"ffn_gate.weight", (uint64_t)H, (uint64_t)F, &w.gu, 0},
        {"ffn_up.weight", (uint64_t)H, (uint64_t)F, &w.gu, F},
        {"ffn_down.weight", (uint64_t)F, (uint64_t)H, &w.down, 0},
    };
    for (auto& q : q8) {
      const char* name = P(q.n);
      const sem_tensor_view* t = find_view(tv, nt, name);
      if ((rc = check_q8(t, name, q.k, q.rows))) return rc;
      if ((rc = upload_q8_proj(ctx, staging, t, (int64_t)q.rows, (int)q.k, *q.w, q.roff))) return rc;
    }
  }
  // ---- the dense head (not read by the reference; the model-faithful mode's) ----
  {
    const sem_tensor_view* t2 = find_view(tv, nt, "dense_2.weight");
    const sem_tensor_view* t3 = find_view(tv, nt, "dense_3.weight");
    if (t2 && t3 && t2->dtype == kQ8 && t3->dtype == kQ8 && t2->n_dims >= 2 && t3->n_dims >= 2 &&
        t2->dims[0] == (uint64_t)H && t3->dims[1] == (uint64_t)H && t3->dims[0] == t2->dims[1] &&
        t2->dims[1] % 128 == 0) {
      const int64_t mid = (int64_t)t2->dims[1];
      size_t doff = 0;
      auto dtake = [&](size_t bytes) {
        size_t o = doff;
        doff = align256(doff + bytes);
        return o;
      };
      struct DOff { size_t codes, scales, hi, rsc, lanes; };
      auto dproj = [&](int64_t rows, int64_t k) {
        DOff p;
        p.codes = dtake((size_t)rows * k * 2);
        p.scales = dtake((size_t)rows * (k / 32) * 4);
        p.hi = dtake((size_t)2 * rows * k * 2);
        p.rsc = dtake((size_t)rows * 4);
        p.lanes = dtake((size_t)rows * k);
        return p;
      };
      const DOff o2 = dproj(mid, H), o3 = dproj(H, mid);
      e = m->dense_buf.ensure(doff);
      if (e != cudaSuccess) return set_error(SEM_ENOMEM, "device allocation of %zu bytes failed: %s", doff, cudaGetErrorString(e));
      uint8_t* db = m->dense_buf.as<uint8_t>();
      auto mk = [&](const DOff& p, int64_t rows, int64_t k) {
        return Q8Proj{reinterpret_cast<const __half*>(db + p.codes), reinterpret_cast<const float*>(db + p.scales),
                      reinterpret_cast<const __half*>(db + p.hi),
                      reinterpret_cast<const __half*>(db + p.hi + (size_t)rows * k * 2),
                      reinterpret_cast<const float*>(db + p.rsc), reinterpret_cast<const int8_t*>(db + p.lanes)};
      };
      m->dense2 = mk(o2, mid, H);
      m->dense3 = mk(o3, H, mid);
      if ((rc = upload_q8_proj(ctx, staging, t2, mid, H, m->dense2, 0))) return rc;
      if ((rc = upload_q8_proj(ctx, staging, t3, H, (int)mid, m->dense3, 0))) return rc;
      m->dense_mid = (int32_t)mid;
    }
  }
  // ---- RoPE tables (rope_cache.go:15-44) ----
  {
    const int half = hd / 2;
    std::vector<float> freqs(half), cs((size_t)c.max_seq_len * half), sn((size_t)c.max_seq_len * half);
    for (int i = 0; i < half; ++i) freqs[i] = (float)(1.0 / std::pow((double)c.rope_base, (double)(2 * i) / (double)hd));
    for (int p = 0; p < c.max_seq_len; ++p)
      for (int i = 0; i < half; ++i) {
        float theta = (float)p * freqs[i];
        cs[(size_t)p * half + i] = (float)std::cos((double)theta);
        sn[(size_t)p * half + i] = (float)std::sin((double)theta);
      }
    SEM_CUDA(cudaMemcpy(m->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
    SEM_CUDA(cudaMemcpy(m->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
  }
  SEM_CUDA(cudaStreamSynchronize(ctx->stream));
  *out = m.release();
  return SEM_OK;
}

// ---------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------
namespace {

int ensure_workspace(sem_model* m, int64_t T, int B, int64_t out_floats) {
  const sem_model_config& c = m->cfg;
  const int H = c.embed_dim, F = c.interm_dim, nh = c.num_heads, hd = c.head_dim;
  const int qkvN = nh * hd + 2 * hd;
  const int64_t Tp = T > 0 ? T : 1;
  SEM_CUDA(m->hid.ensure((size_t)Tp * H * 4));
  SEM_CUDA(m->big.ensure((size_t)Tp * (qkvN > F ? qkvN : F) * 4));
  SEM_CUDA(m->att.ensure((size_t)Tp * H * 4));
  SEM_CUDA(m->codes.ensure((size_t)Tp * (F > H ? F : H) * 2));
  SEM_CUDA(m->halves.ensure((size_t)Tp * (2 * nh * hd + 4 * hd) * 2));
  SEM_CUDA(m->inv_rms.ensure((size_t)Tp * 4));
  // meta: row_seq[T], row_pos[T], cu[B+1], tile_seq/tile_row0[2*(T/64+B)], out_dims[B], out_off (int64) [B],
  // src_row[T]
  size_t meta_ints = (size_t)3 * Tp + (B + 1) + 2 * ((size_t)Tp / 64 + B + 1) + B + 2 * (size_t)B + B +
                     2 * ((size_t)Tp / 256 + B + 1) + 10;
  SEM_CUDA(m->meta.ensure(meta_ints * 4));
  SEM_CUDA(m->absmax.ensure((size_t)(4 * c.num_layers + 1) * (B > 0 ? B : 1) * 4));
  SEM_CUDA(m->ids.ensure((size_t)Tp * 4));
  SEM_CUDA(m->out.ensure((size_t)(out_floats > 0 ? out_floats : 1) * 4));
  // device error words: [0] bad token id seen by the embedding kernel, [1]
  // error bits of a timed-out pipeline wait. They accumulate over forwards
  // until a host read (sem_embed, sem_model_check) clears them.
  if (m->faithful.dense_head) {
    SEM_CUDA(m->head_y1.ensure((size_t)(B > 0 ? B : 1) * m->dense_mid * 4));
    SEM_CUDA(m->head_codes.ensure((size_t)(B > 0 ? B : 1) * m->dense_mid * 2));
    SEM_CUDA(m->head_absmax.ensure((size_t)2 * (B > 0 ? B : 1) * 4));
  }
  const bool new_flags = m->errflag.bytes < 16;
  SEM_CUDA(m->errflag.ensure(16));
  if (new_flags) SEM_CUDA(cudaMemsetAsync(m->errflag.p, 0, 16, m->ctx->stream));
  return SEM_OK;
}

struct MetaPtrs {
  SeqMeta seq;
  AttnTiles tiles;        // 128-row attention tiles of the long sequences (tensor-core kernel)
  AttnTiles short_tiles;  // one tile per short sequence (float32 CUDA-core kernel)
  AttnTiles pair_tiles;   // 256-row tiles of the long sequences (SM-pair tensor-core kernel)
  AttnTiles pair_all;     // 256-row tiles of every sequence
  int32_t short_max_len;  // longest short sequence
  int32_t* out_dims;
  int64_t* out_off;
  const int32_t* iota;  // [B] 0, 1, ..., B - 1 (one quantisation scale per pooled row)
  int32_t* src_row;  // [T] caller's row of each packed row (valid when permuted)
  int64_t T_long;    // packed rows [0, T_long) belong to sequences of >= kSplitMinLen tokens
  bool permuted;     // the packed order differs from the caller's
};

// Sequences at least this long take the tensor-core kernels: the split-plane
// projections (block scales folded into the weights; their GEMM outputs differ
// from the reference's per-block float32 sums in the last bits only, which
// mean pooling over many tokens keeps within the reference's own spread
// between its builds) and the split-fp16 tensor-core attention. Shorter
// sequences take the CUDA-core projection and attention kernels, whose float32
// operations are the reference's in the reference's order: their embeddings
// are bit-identical to the reference's default build.
constexpr int32_t kSplitMinLen = 128;
// Up to this many tokens of short sequences in a batch take the exact
// kernels under SEM_Q8_PATH_AUTO (the latency regime of small requests).
constexpr int64_t kExactShortMaxTokens = 4096;

// Builds the per-batch metadata on the host and uploads it (skipped when the
// batch shape equals the previous call's). Sequences are packed long ones
// (>= kSplitMinLen tokens) first, each group in the caller's order; the
// outputs go back to the caller's order through out_off.
int upload_meta(sem_model* m, const int32_t* offsets, int B, const int32_t* dims, MetaPtrs* mp,
                HostBuf* staging = nullptr) {
  const int64_t T = offsets[B];
  int32_t* base = m->meta.as<int32_t>();
  int32_t* d_row_seq = base;
  int32_t* d_row_pos = d_row_seq + T;
  int32_t* d_cu = d_row_pos + T;
  int64_t max_tiles = T / 64 + B + 1;
  int32_t* d_tseq = d_cu + (B + 1);
  int32_t* d_trow = d_tseq + max_tiles;
  int32_t* d_dims = d_trow + max_tiles;
  int32_t* d_src = d_dims + B;
  uintptr_t p = reinterpret_cast<uintptr_t>(d_src + T);
  p = (p + 7) & ~uintptr_t(7);
  int64_t* d_off = reinterpret_cast<int64_t*>(p);
  int32_t* d_iota = reinterpret_cast<int32_t*>(d_off + B);
  const int64_t max_ptiles = T / 256 + B + 1;
  int32_t* d_pseq = d_iota + B;
  int32_t* d_prow = d_pseq + max_ptiles;
  bool same = (int)m->last_offsets.size() == B + 1 &&
              std::memcmp(m->last_offsets.data(), offsets, sizeof(int32_t) * (B + 1)) == 0 &&
              (int)m->last_dims.size() == B && std::memcmp(m->last_dims.data(), dims, sizeof(int32_t) * B) == 0;
  if (!same) {
    // packed order: long sequences, then short ones (stable)
    std::vector<int32_t> order;
    order.reserve(B);
    int64_t t_long = 0;
    for (int s = 0; s < B; ++s)
      if (offsets[s + 1] - offsets[s] >= kSplitMinLen) {
        order.push_back(s);
        t_long += offsets[s + 1] - offsets[s];
      }
    for (int s = 0; s < B; ++s)
      if (offsets[s + 1] - offsets[s] < kSplitMinLen) order.push_back(s);
    bool permuted = false;
    for (int s = 0; s < B; ++s) permuted |= order[s] != s;
    std::vector<int64_t> caller_off(B);
    int64_t acc = 0;
    for (int s = 0; s < B; ++s) {
      caller_off[s] = acc;
      acc += dims[s];
    }
    size_t bytes = (size_t)(reinterpret_cast<uint8_t*>(d_prow + max_ptiles) - reinterpret_cast<uint8_t*>(base));
    // a request slot's own staging is free (its previous request completed);
    // the shared pinned buffer may still feed an earlier copy
    HostBuf& hb = staging ? *staging : m->ctx->pinned;
    if (!staging) SEM_CUDA(cudaStreamSynchronize(m->ctx->stream));
    SEM_CUDA(hb.ensure(bytes));
    int32_t* h = hb.as<int32_t>();
    int32_t* h_row_seq = h;
    int32_t* h_row_pos = h_row_seq + T;
    int32_t* h_cu = h_row_pos + T;
    int32_t* h_tseq = h_cu + (B + 1);
    int32_t* h_trow = h_tseq + max_tiles;
    int32_t* h_dims = h_trow + max_tiles;
    int32_t* h_src = h_dims + B;
    int64_t* h_off = reinterpret_cast<int64_t*>(reinterpret_cast<uint8_t*>(h) +
                                                (reinterpret_cast<uint8_t*>(d_off) - reinterpret_cast<uint8_t*>(base)));
    int32_t* h_iota = reinterpret_cast<int32_t*>(h_off + B);
    int32_t* h_pseq = h_iota + B;
    int32_t* h_prow = h_pseq + max_ptiles;
    for (int s = 0; s < B; ++s) h_iota[s] = s;
    int32_t nt = 0, nt_long = 0, short_max = 0, np = 0, np_long = 0;
    int32_t r = 0;
    for (int s = 0; s < B; ++s) {
      const int o = order[s];
      const int32_t len = offsets[o + 1] - offsets[o];
      if (len >= kSplitMinLen) nt_long = nt + (len + kAttnTileRows - 1) / kAttnTileRows;
      else if (len > short_max) short_max = len;
      h_cu[s] = r;
      for (int32_t i = 0; i < len; ++i) {
        h_row_seq[r + i] = s;
        h_row_pos[r + i] = i;
        h_src[r + i] = offsets[o] + i;
      }
      for (int32_t i = 0; i < len; i += kAttnTileRows) {
        h_tseq[nt] = s;
        h_trow[nt] = r + i;
        ++nt;
      }
      for (int32_t i = 0; i < len; i += 2 * kAttnTileRows) {
        h_pseq[np] = s;
        h_prow[np] = r + i;
        ++np;
      }
      if (len >= kSplitMinLen) np_long = np;
      h_dims[s] = dims[o];
      h_off[s] = caller_off[o];
      r += len;
    }
    h_cu[B] = r;
    SEM_CUDA(cudaMemcpyAsync(base, h, bytes, cudaMemcpyHostToDevice, m->ctx->stream));
    m->last_offsets.assign(offsets, offsets + B + 1);
    m->last_dims.assign(dims, dims + B);
    m->n_tiles = nt;
    m->n_tiles_long = nt_long;
    m->n_ptiles = np;
    m->n_ptiles_long = np_long;
    m->short_max_len = short_max;
    m->t_long = t_long;
    m->permuted = permuted;
  }
  mp->seq = SeqMeta{d_row_seq, d_row_pos, d_cu, (int32_t)T, (int32_t)B};
  mp->tiles = AttnTiles{d_tseq, d_trow, m->n_tiles_long};
  mp->short_max_len = m->short_max_len;
  mp->short_tiles = AttnTiles{d_tseq + m->n_tiles_long, d_trow + m->n_tiles_long, m->n_tiles - m->n_tiles_long};
  // SM-pair attention (256-row tiles) unless sequences of 128-255 tokens would
  // leave more than a quarter of its CTAs without rows: then 128-row tiles
  const bool pairs_long = 8 * m->n_ptiles_long <= 5 * m->n_tiles_long;
  const bool pairs_all = 8 * m->n_ptiles <= 5 * m->n_tiles;
  mp->pair_tiles = AttnTiles{d_pseq, d_prow, pairs_long ? m->n_ptiles_long : 0};
  mp->pair_all = AttnTiles{d_pseq, d_prow, pairs_all ? m->n_ptiles : 0};
  mp->out_dims = d_dims;
  mp->out_off = d_off;
  mp->iota = d_iota;
  mp->src_row = d_src;
  mp->T_long = m->t_long;
  mp->permuted = m->permuted;
  return SEM_OK;
}

// Stage ids for the optional per-launch timing (sem_model_profile).
enum Stage { kStEmbed, kStRowStats, kStQuant, kStGemmQKV, kStQKNormRope, kStAttention, kStGemmO, kStResidual,
             kStGemmGateUp, kStGemmDown, kStPool, kStAttnShort, kStages };
const char* const kStageNames[kStages] = {"embed", "row_stats", "quantize", "gemm_q8_qkv", "qk_norm_rope", "attention",
                                          "gemm_q8_o", "residual_norm", "gemm_q8_gate_up", "gemm_q8_down", "pool_l2",
                                          "attention_short"};

}  // namespace

// Records an event before a launch when profiling (bracketing pairs).
void prof_mark(sem_model* m, int stage, cudaStream_t st, bool after);

namespace {

#define SEM_LAUNCH(stage, call)                                                                 \
  do {                                                                                          \
    if (m->prof) prof_mark(m, (stage), st, false);                                              \
    cudaError_t e_ = (call);                                                                    \
    if (e_ != cudaSuccess) return set_error(SEM_EDEVICE, "forward: %s", cudaGetErrorString(e_)); \
    if (m->prof) prof_mark(m, (stage), st, true);                                               \
  } while (0)

// The whole forward on `st`: ids already on the device in m->ids (or d_ids).
int run_forward(sem_model* m, const int32_t* d_ids, const MetaPtrs& mp, float* d_out, cudaStream_t st) {
  const sem_model_config& c = m->cfg;
  const int H = c.embed_dim, F = c.interm_dim, L = c.num_layers, nh = c.num_heads, hd = c.head_dim;
  const int qkvN = nh * hd + 2 * hd;
  const SeqMeta& sm = mp.seq;
  const int64_t T = sm.T;
  const int B = sm.B;
  float* hid = m->hid.as<float>();
  float* big = m->big.as<float>();
  float* att = m->att.as<float>();
  __half* codes = m->codes.as<__half>();
  uint32_t* err = m->errflag.as<uint32_t>() + 1;
  float* inv = m->inv_rms.as<float>();
  uint32_t* amax = m->absmax.as<uint32_t>();
  __half* hb = m->halves.as<__half>();
  __half *qh = hb, *ql = qh + T * nh * hd, *kh = ql + T * nh * hd, *kl = kh + T * hd, *vh = kl + T * hd,
         *vl = vh + T * hd;
  auto slot = [&](int l, int k) { return amax + (size_t)(4 * l + k) * B; };
  // Q8_0 projection of all packed rows: rows [0, t_split) (long sequences)
  // through launch_q8_proj, the rest (short sequences) through the CUDA-core
  // VNNI-order kernel, or the per-block tensor-core kernel under path 1.
  // out_cols: columns of one output row (N, or N / 2 for gate/up).
  const int q8_path = get_q8_path();
  const int64_t t_split = q8_path == 3 || q8_path == 4 ? T : q8_path == 1 ? 0 : mp.T_long;
  // Short sequences take the exact kernels (bit-identical to the reference)
  // under path 4, and under path 0 while their tokens are few enough for the
  // CUDA cores to match the tensor cores' latency; otherwise the tensor-core
  // projection and attention kernels, as long sequences do.
  const bool exact_short = q8_path == 4 || (q8_path == 0 && T - mp.T_long <= kExactShortMaxTokens);
  auto q8 = [&](const Q8Proj& w, int N, int K, const uint32_t* a_absmax, float* out, int out_cols, int epi,
                uint32_t* out_absmax, const VPlanes& vp = VPlanes{}) -> cudaError_t {
    cudaError_t e = cudaSuccess;
    if (t_split > 0)
      e = launch_q8_proj(codes, w, (int)t_split, N, K, a_absmax, sm.row_seq, out, epi, out_absmax, err, st, vp);
    if (e == cudaSuccess && T > t_split) {
      if (!exact_short)
        e = launch_gemm_q8(codes + t_split * K, w.codes, w.scales, (int)(T - t_split), N, K, a_absmax,
                           sm.row_seq + t_split, out + t_split * out_cols, epi, out_absmax, err, st);
      else
        e = launch_gemm_q8_dp4a(codes + t_split * K, w.lanes, w.scales, (int)(T - t_split), N, K, a_absmax,
                                sm.row_seq + t_split, out + t_split * out_cols, epi, out_absmax, st);
    }
    return e;
  };
  SEM_LAUNCH(kStEmbed, cudaMemsetAsync(amax, 0, (size_t)(4 * L + 1) * B * 4, st));
  SEM_LAUNCH(kStEmbed, launch_embed(d_ids, m->emb, m->emb_s, c.vocab_size, H, hid, (int)T, m->errflag.as<uint32_t>(), st));
  SEM_LAUNCH(kStRowStats, launch_row_stats(hid, m->layers[0].attn_norm, H, c.norm_eps, sm, inv, slot(0, 0), st));
  // the first attention norm's codes; every later norm is quantized by the
  // residual kernel before it
  SEM_LAUNCH(kStQuant, launch_quantize(hid, inv, m->layers[0].attn_norm, H, sm, slot(0, 0), codes, st));
  const sem_faithful_config& fa = m->faithful;
  const float* swa_cos = m->rope_swa.p ? m->rope_swa.as<float>() : m->rope_cos;
  const float* swa_sin = m->rope_swa.p ? m->rope_swa.as<float>() + (size_t)c.max_seq_len * (hd / 2) : m->rope_sin;
  for (int l = 0; l < L; ++l) {
    const LayerW& w = m->layers[l];
    // model-faithful mode: sliding layers (all but every swa_pattern-th) see
    // keys within sliding_window / 2 positions, with their own RoPE tables;
    // otherwise every layer attends to every key (model_int8.go:500)
    const bool sliding = fa.sliding_window > 0 && fa.swa_pattern > 0 && (l + 1) % fa.swa_pattern != 0;
    const int hw = sliding ? fa.sliding_window / 2 : 0;
    // attention block (model_int8.go:191-210)
    // the long rows' V columns go straight to the attention's hi / lo planes
    // when the split-plane kernel projects them (v_planes: it did)
    bool v_planes = false;
    SEM_LAUNCH(kStGemmQKV, q8(w.qkv, qkvN, H, slot(l, 0), big, qkvN, kEpiStore, nullptr,
                              VPlanes{vh, T, nh * hd + hd, &v_planes}));
    SEM_LAUNCH(kStQKNormRope, launch_qk_norm_rope(big, w.q_norm, w.k_norm, sliding ? swa_cos : m->rope_cos,
                                                  sliding ? swa_sin : m->rope_sin, c.norm_eps, nh, sm, qh, ql, kh, kl,
                                                  vh, vl, exact_short ? mp.T_long : T,
                                                  v_planes ? t_split : 0, st));
    if (exact_short) {  // tensor cores for the long sequences' tiles, float32 CUDA cores for the short ones
      if (mp.tiles.n_tiles)
        SEM_LAUNCH(kStAttention, launch_attention(qh, ql, kh, kl, vh, vl, nh, c.attention_scale, hw, sm, mp.tiles,
                                                  mp.pair_tiles, att, slot(l, 1), err, st));
      if (mp.short_tiles.n_tiles)
        SEM_LAUNCH(kStAttnShort, launch_attention_short(big, nh, c.attention_scale, hw, sm, mp.short_tiles,
                                                        mp.short_max_len, att, slot(l, 1), st));
    } else {
      const AttnTiles all{mp.tiles.tile_seq, mp.tiles.tile_row0, mp.tiles.n_tiles + mp.short_tiles.n_tiles};
      SEM_LAUNCH(kStAttention, launch_attention(qh, ql, kh, kl, vh, vl, nh, c.attention_scale, hw, sm, all,
                                                mp.pair_all, att, slot(l, 1), err, st));
    }
    SEM_LAUNCH(kStQuant, launch_quantize(att, nullptr, nullptr, H, sm, slot(l, 1), codes, st));
    SEM_LAUNCH(kStGemmO, q8(w.o, H, H, slot(l, 1), big, H, kEpiStore, nullptr));
    SEM_LAUNCH(kStResidual, launch_residual_norm(big, w.post_attn, hid, w.ffn_norm, H, c.norm_eps, sm, inv, slot(l, 2),
                                                 codes, st));
    // MLP block (model_int8.go:213-232)
    SEM_LAUNCH(kStGemmGateUp, q8(w.gu, 2 * F, H, slot(l, 2), big, F, kEpiGeluUp, slot(l, 3)));
    SEM_LAUNCH(kStQuant, launch_quantize(big, nullptr, nullptr, F, sm, slot(l, 3), codes, st));
    SEM_LAUNCH(kStGemmDown, q8(w.down, H, F, slot(l, 3), att, H, kEpiStore, nullptr));
    const bool last = l + 1 == L;
    const float* next_w = last ? m->out_norm : m->layers[l + 1].attn_norm;
    SEM_LAUNCH(kStResidual, launch_residual_norm(att, w.post_ffw, hid, next_w ? next_w : w.ffn_norm, H, c.norm_eps, sm, inv,
                                                 last ? nullptr : slot(l + 1, 0), last ? nullptr : codes, st));
  }
  if (fa.dense_head) {
    // model-faithful head: output_norm + mean pool of every channel, dense_2
    // then dense_3 (each input quantised per sequence like every projection,
    // on the kernel in the reference's VNNI order), then the first dims and L2
    const int mid = m->dense_mid;
    float* pooled = att;  // [B][H]
    float* y1 = m->head_y1.as<float>();
    __half* hc = m->head_codes.as<__half>();
    uint32_t* ha = m->head_absmax.as<uint32_t>();
    SEM_LAUNCH(kStPool, launch_pool_l2(hid, m->out_norm ? inv : nullptr, m->out_norm, H, sm, nullptr, nullptr, pooled,
                                       st));
    SEM_LAUNCH(kStPool, launch_quantize_rows(pooled, B, H, ha, hc, st));
    SEM_LAUNCH(kStPool, launch_gemm_q8_dp4a(hc, m->dense2.lanes, m->dense2.scales, B, mid, H, ha, mp.iota, y1,
                                            kEpiStore, nullptr, st));
    SEM_LAUNCH(kStPool, launch_quantize_rows(y1, B, mid, ha + B, hc, st));
    SEM_LAUNCH(kStPool, launch_gemm_q8_dp4a(hc, m->dense3.lanes, m->dense3.scales, B, H, mid, ha + B, mp.iota, pooled,
                                            kEpiStore, nullptr, st));
    SEM_LAUNCH(kStPool, launch_l2_rows(pooled, B, H, mp.out_dims, mp.out_off, d_out, st));
    return SEM_OK;
  }
  // output_norm + mean pool + L2 (model_int8.go:235-255)
  SEM_LAUNCH(kStPool, launch_pool_l2(hid, m->out_norm ? inv : nullptr, m->out_norm, H, sm, mp.out_dims, mp.out_off, d_out, st));
  return SEM_OK;
}

// Batches up to this many tokens replay a CUDA graph of the forward when the
// shape repeats: their ~240 launches would otherwise cost about as much as
// the kernels' work.
constexpr int64_t kGraphMaxTokens = 32768;

constexpr size_t kGraphCacheSize = 8;

void drop_graphs(sem_model* m) {
  for (auto& g : m->graphs)
    if (g.exec) cudaGraphExecDestroy(g.exec);
  m->graphs.clear();
}

// run_forward on the workspace ids and output, through a graph captured on
// the first call of a small batch shape and replayed while the shape, the
// workspace buffers, the projection path, the mode and the stream stay the
// same. Up to kGraphCacheSize shapes keep their graphs.
int forward_maybe_graph(sem_model* m, const MetaPtrs& mp, const int32_t* offsets, const int32_t* dims,
                        cudaStream_t st) {
  const int64_t T = mp.seq.T;
  const int B = mp.seq.B;
  auto direct = [&] { return run_forward(m, m->ids.as<int32_t>(), mp, m->out.as<float>(), st); };
  if (m->prof || m->graphs_off || T > kGraphMaxTokens) return direct();
  const std::vector<const void*> key = {m->hid.p,    m->big.p,   m->att.p, m->codes.p, m->halves.p,
                                        m->inv_rms.p, m->meta.p,  m->absmax.p, m->ids.p, m->out.p,
                                        m->errflag.p, reinterpret_cast<const void*>((intptr_t)get_q8_path()),
                                        static_cast<const void*>(st),
                                        reinterpret_cast<const void*>((intptr_t)m->faithful_gen), m->head_y1.p};
  std::vector<int32_t> shape(offsets, offsets + B + 1);
  shape.insert(shape.end(), dims, dims + B);
  // graphs of other buffers (the workspace grew) can never replay again
  for (size_t i = 0; i < m->graphs.size();)
    if (m->graphs[i].key != key) {
      cudaGraphExecDestroy(m->graphs[i].exec);
      m->graphs.erase(m->graphs.begin() + i);
    } else {
      ++i;
    }
  sem_model::Graph* hit = nullptr;
  for (auto& g : m->graphs)
    if (g.shape == shape) hit = &g;
  if (!hit) {
    // A capture that the runtime refuses (the kernels were recorded, not run)
    // turns graphs off for this model and runs the same kernels directly; an
    // error of the forward itself is returned as it is.
    if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
      cudaGetLastError();
      m->graphs_off = true;
      return direct();
    }
    const int rc = direct();
    cudaGraph_t g = nullptr;
    const cudaError_t e = cudaStreamEndCapture(st, &g);
    if (e != cudaSuccess || !g) {
      if (g) cudaGraphDestroy(g);
      cudaGetLastError();
      m->graphs_off = true;
      return direct();
    }
    if (rc) {
      cudaGraphDestroy(g);
      return rc;
    }
    cudaGraphExec_t exec = nullptr;
    const cudaError_t ei = cudaGraphInstantiate(&exec, g, 0);
    cudaGraphDestroy(g);
    if (ei != cudaSuccess) {
      cudaGetLastError();
      m->graphs_off = true;
      return direct();
    }
    if (m->graphs.size() >= kGraphCacheSize) {
      auto lru = std::min_element(m->graphs.begin(), m->graphs.end(),
                                  [](const sem_model::Graph& a, const sem_model::Graph& b) { return a.used < b.used; });
      cudaGraphExecDestroy(lru->exec);
      m->graphs.erase(lru);
    }
    m->graphs.push_back(sem_model::Graph{key, std::move(shape), exec, 0});
    hit = &m->graphs.back();
  }
  hit->used = ++m->graph_tick;
  SEM_CUDA(cudaGraphLaunch(hit->exec, st));
  return SEM_OK;
}

}  // namespace

int validate_embed_request(const sem_model_config& c, const int32_t* ids, const int32_t* offsets, int32_t B,
                           const int32_t* dims_in, float* out, std::vector<int32_t>* dims, int64_t* out_floats) {
  if ((!ids && B > 0) || !offsets || (!out && B > 0)) return set_error(SEM_EINVAL, "null argument");
  if (B < 0) return set_error(SEM_EINVAL, "negative sequence count");
  if (B > 0 && offsets[0] != 0) return set_error(SEM_EINVAL, "offsets[0] must be 0");
  dims->assign(B, 0);
  *out_floats = 0;
  for (int s = 0; s < B; ++s) {
    int d = dims_in ? dims_in[s] : c.embed_dim;
    // ForwardWithDim (model.go:661-666) then forwardINT8WithDim (model_int8.go:149-171)
    if (d <= 0 || d > c.embed_dim)
      return set_error(SEM_EINVAL, "target dimension %d out of range (1..%d)", d, c.embed_dim);
    int len = offsets[s + 1] - offsets[s];
    if (len <= 0) return set_error(SEM_EINVAL, "empty input");
    if (len > c.max_seq_len) return set_error(SEM_EINVAL, "sequence too long: %d > %d", len, c.max_seq_len);
    for (int32_t r = offsets[s]; r < offsets[s + 1]; ++r)
      if (ids[r] < 0 || ids[r] >= c.vocab_size) return set_error(SEM_EINVAL, "token ID out of range: %d", ids[r]);
    (*dims)[s] = d;
    *out_floats += d;
  }
  return SEM_OK;
}

int model_embed(sem_model* m, const int32_t* ids, const int32_t* offsets, int32_t B, const int32_t* dims_in,
                float* out) {
  if (!m) return set_error(SEM_EINVAL, "null argument");
  std::vector<int32_t> dims;
  int64_t out_floats = 0;
  if (int rc = validate_embed_request(m->cfg, ids, offsets, B, dims_in, out, &dims, &out_floats)) return rc;
  if (B == 0) return SEM_OK;
  sem_context* ctx = m->ctx;
  DeviceGuard dg(ctx->device);
  std::lock_guard<std::mutex> lk(ctx->mu);
  const int64_t T = offsets[B];
  int rc;
  if ((rc = ensure_workspace(m, T, B, out_floats))) return rc;
  MetaPtrs mp;
  if ((rc = upload_meta(m, offsets, B, dims.data(), &mp))) return rc;
  if (mp.permuted) {  // ids in the packed order (long sequences first)
    SEM_CUDA(m->ids_in.ensure((size_t)T * 4));
    SEM_CUDA(cudaMemcpyAsync(m->ids_in.p, ids, (size_t)T * 4, cudaMemcpyHostToDevice, ctx->stream));
    SEM_CUDA(launch_gather_i32(m->ids_in.as<int32_t>(), mp.src_row, m->ids.as<int32_t>(), T, ctx->stream));
  } else {
    SEM_CUDA(cudaMemcpyAsync(m->ids.p, ids, (size_t)T * 4, cudaMemcpyHostToDevice, ctx->stream));
  }
  if ((rc = forward_maybe_graph(m, mp, offsets, dims.data(), ctx->stream))) return rc;
  SEM_CUDA(cudaMemcpyAsync(out, m->out.p, (size_t)out_floats * 4, cudaMemcpyDeviceToHost, ctx->stream));
  SEM_CUDA(ctx->pinned.ensure(64));
  uint32_t* flags = ctx->pinned.as<uint32_t>();
  SEM_CUDA(cudaMemcpyAsync(flags, m->errflag.p, 8, cudaMemcpyDeviceToHost, ctx->stream));
  SEM_CUDA(cudaMemsetAsync(m->errflag.p, 0, 8, ctx->stream));
  SEM_CUDA(cudaStreamSynchronize(ctx->stream));
  if (flags[1]) return set_error(SEM_EDEVICE, "forward: a tensor-core pipeline wait timed out (error bits 0x%x)", flags[1]);
  return SEM_OK;
}

// The request pipeline: submit validates a request, stages its ids and
// metadata in a slot's pinned buffers and enqueues the upload, the forward and
// the download of its outputs and error words, then returns; wait blocks on
// that request alone and hands its outputs over. With two slots the host
// prepares (and tokenises) request i + 1 while the device runs request i, the
// overlap the reference gets from one goroutine per prompt
// (pkg/ggufembed/api.go:237-295).
int model_embed_submit(sem_model* m, const int32_t* ids, const int32_t* offsets, int32_t B, const int32_t* dims_in,
                       uint64_t* ticket) {
  if (!m || !ticket) return set_error(SEM_EINVAL, "null argument");
  std::vector<int32_t> dims;
  int64_t out_floats = 0;
  float dummy = 0.0f;
  if (int rc = validate_embed_request(m->cfg, ids, offsets, B, dims_in, &dummy, &dims, &out_floats)) return rc;
  sem_context* ctx = m->ctx;
  DeviceGuard dg(ctx->device);
  std::lock_guard<std::mutex> lk(ctx->mu);
  sem_model::Slot& sl = m->slots[m->next_ticket & 1];
  if (sl.busy) return set_error(SEM_EINVAL, "two requests in flight: wait for one before submitting another");
  if (!sl.done) SEM_CUDA(cudaEventCreateWithFlags(&sl.done, cudaEventDisableTiming));
  SEM_CUDA(sl.flags.ensure(64));
  uint32_t* flags = sl.flags.as<uint32_t>();
  flags[0] = flags[1] = 0;
  sl.out_floats = out_floats;
  auto enqueue = [&]() -> int {
    if (B == 0) return SEM_OK;
    const int64_t T = offsets[B];
    int rc;
    if ((rc = ensure_workspace(m, T, B, out_floats))) return rc;
    MetaPtrs mp;
    if ((rc = upload_meta(m, offsets, B, dims.data(), &mp, &sl.meta))) return rc;
    SEM_CUDA(sl.ids.ensure((size_t)T * 4));
    SEM_CUDA(sl.out.ensure((size_t)out_floats * 4));
    std::memcpy(sl.ids.p, ids, (size_t)T * 4);
    if (mp.permuted) {
      SEM_CUDA(m->ids_in.ensure((size_t)T * 4));
      SEM_CUDA(cudaMemcpyAsync(m->ids_in.p, sl.ids.p, (size_t)T * 4, cudaMemcpyHostToDevice, ctx->stream));
      SEM_CUDA(launch_gather_i32(m->ids_in.as<int32_t>(), mp.src_row, m->ids.as<int32_t>(), T, ctx->stream));
    } else {
      SEM_CUDA(cudaMemcpyAsync(m->ids.p, sl.ids.p, (size_t)T * 4, cudaMemcpyHostToDevice, ctx->stream));
    }
    if ((rc = forward_maybe_graph(m, mp, offsets, dims.data(), ctx->stream))) return rc;
    SEM_CUDA(cudaMemcpyAsync(sl.out.p, m->out.p, (size_t)out_floats * 4, cudaMemcpyDeviceToHost, ctx->stream));
    SEM_CUDA(cudaMemcpyAsync(flags, m->errflag.p, 8, cudaMemcpyDeviceToHost, ctx->stream));
    SEM_CUDA(cudaMemsetAsync(m->errflag.p, 0, 8, ctx->stream));
    return SEM_OK;
  };
  if (int rc = enqueue()) {
    // part of the request may be enqueued already and still read the
    // slot's pinned buffers: let it finish before the slot is reused
    cudaStreamSynchronize(ctx->stream);
    return rc;
  }
  SEM_CUDA(cudaEventRecord(sl.done, ctx->stream));
  sl.busy = true;
  sl.ticket = m->next_ticket++;
  *ticket = sl.ticket;
  return SEM_OK;
}

int model_embed_wait(sem_model* m, uint64_t ticket, float* out) {
  if (!m) return set_error(SEM_EINVAL, "null argument");
  sem_context* ctx = m->ctx;
  DeviceGuard dg(ctx->device);
  sem_model::Slot* sl = nullptr;
  cudaEvent_t ev = nullptr;
  {
    std::lock_guard<std::mutex> lk(ctx->mu);
    for (auto& x : m->slots)
      if (x.busy && x.ticket == ticket) sl = &x;
    if (!sl) return set_error(SEM_EINVAL, "no request in flight with ticket %llu", (unsigned long long)ticket);
    if (!out && sl->out_floats > 0) return set_error(SEM_EINVAL, "null argument");
    ev = sl->done;
  }
  // outside the lock: the other slot's submit may enqueue meanwhile
  const cudaError_t es = cudaEventSynchronize(ev);
  std::lock_guard<std::mutex> lk(ctx->mu);
  sl->busy = false;
  if (es != cudaSuccess) return set_error(SEM_EDEVICE, "cudaEventSynchronize: %s", cudaGetErrorString(es));
  const uint32_t* flags = sl->flags.as<uint32_t>();
  if (flags[1]) return set_error(SEM_EDEVICE, "forward: a tensor-core pipeline wait timed out (error bits 0x%x)", flags[1]);
  if (sl->out_floats > 0) std::memcpy(out, sl->out.p, (size_t)sl->out_floats * 4);
  return SEM_OK;
}

int model_set_faithful(sem_model* m, const sem_faithful_config* f) {
  if (!m) return set_error(SEM_EINVAL, "null argument");
  sem_faithful_config cfg{};
  if (f) cfg = *f;
  if (cfg.sliding_window < 0 || cfg.swa_pattern < 0 || cfg.rope_base_swa < 0.0f)
    return set_error(SEM_EINVAL, "faithful mode: negative sliding_window, swa_pattern or rope_base_swa");
  if (cfg.dense_head && !m->dense_mid)
    return set_error(SEM_EINVAL, "faithful mode: the model has no dense_2.weight / dense_3.weight to apply");
  sem_context* ctx = m->ctx;
  DeviceGuard dg(ctx->device);
  std::lock_guard<std::mutex> lk(ctx->mu);
  SEM_CUDA(cudaStreamSynchronize(ctx->stream));
  const sem_model_config& c = m->cfg;
  DevBuf table;  // built before anything changes: a failure leaves the model's setting and tables as they were
  if (cfg.sliding_window > 0 && cfg.rope_base_swa > 0.0f && cfg.rope_base_swa != c.rope_base) {
    // rope_cache.go:15-44 with the sliding layers' base
    const int half = c.head_dim / 2;
    std::vector<float> freqs(half), tab((size_t)2 * c.max_seq_len * half);
    for (int i = 0; i < half; ++i)
      freqs[i] = (float)(1.0 / std::pow((double)cfg.rope_base_swa, (double)(2 * i) / (double)c.head_dim));
    for (int p = 0; p < c.max_seq_len; ++p)
      for (int i = 0; i < half; ++i) {
        const float theta = (float)p * freqs[i];
        tab[(size_t)p * half + i] = (float)std::cos((double)theta);
        tab[(size_t)c.max_seq_len * half + (size_t)p * half + i] = (float)std::sin((double)theta);
      }
    SEM_CUDA(table.ensure(tab.size() * 4));
    SEM_CUDA(cudaMemcpy(table.p, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice));
  }
  std::swap(m->rope_swa.p, table.p);  // the old table is freed with `table`
  std::swap(m->rope_swa.bytes, table.bytes);
  m->faithful = cfg;
  ++m->faithful_gen;
  return SEM_OK;
}

sem_faithful_config model_faithful_get(const sem_model* m) { return m->faithful; }

int model_check(sem_model* m) {
  if (!m) return set_error(SEM_EINVAL, "null argument");
  sem_context* ctx = m->ctx;
  DeviceGuard dg(ctx->device);
  std::lock_guard<std::mutex> lk(ctx->mu);
  // forwards may have been enqueued on caller streams (sem_embed_device)
  SEM_CUDA(cudaDeviceSynchronize());
  if (!m->errflag.p) return SEM_OK;
  SEM_CUDA(ctx->pinned.ensure(64));
  uint32_t* flags = ctx->pinned.as<uint32_t>();
  SEM_CUDA(cudaMemcpyAsync(flags, m->errflag.p, 8, cudaMemcpyDeviceToHost, ctx->stream));
  SEM_CUDA(cudaMemsetAsync(m->errflag.p, 0, 8, ctx->stream));
  SEM_CUDA(cudaStreamSynchronize(ctx->stream));
  if (flags[1]) return set_error(SEM_EDEVICE, "forward: a tensor-core pipeline wait timed out (error bits 0x%x)", flags[1]);
  if (flags[0])
    return set_error(SEM_EINVAL, "token ID out of range: a device-resident id outside [0, %d)", m->cfg.vocab_size);
  return SEM_OK;
}

int model_embed_device(sem_model* m, const int32_t* d_ids, const int32_t* h_offsets, int32_t B, int32_t dim,
                       float* d_out, void* stream) {
  if (!m || !d_ids || !h_offsets || !d_out) return set_error(SEM_EINVAL, "null argument");
  const sem_model_config& c = m->cfg;
  if (dim <= 0 || dim > c.embed_dim) return set_error(SEM_EINVAL, "target dimension %d out of range (1..%d)", dim, c.embed_dim);
  for (int s = 0; s < B; ++s) {
    int len = h_offsets[s + 1] - h_offsets[s];
    if (len <= 0) return set_error(SEM_EINVAL, "empty input");
    if (len > c.max_seq_len) return set_error(SEM_EINVAL, "sequence too long: %d > %d", len, c.max_seq_len);
  }
  if (B == 0) return SEM_OK;
  sem_context* ctx = m->ctx;
  DeviceGuard dg(ctx->device);
  std::lock_guard<std::mutex> lk(ctx->mu);
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  std::vector<int32_t> dims(B, dim);
  int rc;
  if ((rc = ensure_workspace(m, h_offsets[B], B, (int64_t)B * dim))) return rc;
  MetaPtrs mp;
  if ((rc = upload_meta(m, h_offsets, B, dims.data(), &mp))) return rc;
  if (st != ctx->stream) {  // metadata was uploaded on the context stream
    cudaEvent_t ev;
    SEM_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    SEM_CUDA(cudaEventRecord(ev, ctx->stream));
    SEM_CUDA(cudaStreamWaitEvent(st, ev, 0));
    cudaEventDestroy(ev);
  }
  if (mp.permuted) {  // ids in the packed order (long sequences first)
    SEM_CUDA(launch_gather_i32(d_ids, mp.src_row, m->ids.as<int32_t>(), h_offsets[B], st));
    d_ids = m->ids.as<int32_t>();
  }
  return run_forward(m, d_ids, mp, d_out, st);
}

// ---------------------------------------------------------------------------
// Isolated Q8_0 projection (config-2 microbench)
// ---------------------------------------------------------------------------
int q8_weight_create(sem_context* ctx, const void* w_q8, int32_t k_in, int32_t n_out, sem_q8_weight** out) {
  if (!ctx || !w_q8 || !out) return set_error(SEM_EINVAL, "null argument");
  if (k_in <= 0 || n_out <= 0 || k_in % 128 || n_out % 128)
    return set_error(SEM_EINVAL, "q8 weight %d x %d: both dimensions must be positive multiples of 128", k_in, n_out);
  DeviceGuard dg(ctx->device);
  std::lock_guard<std::mutex> lk(ctx->mu);
  std::unique_ptr<sem_q8_weight> w(new sem_q8_weight());
  w->ctx = ctx;
  w->k_in = k_in;
  w->n_out = n_out;
  SEM_CUDA(w->codes.ensure((size_t)k_in * n_out * 2));
  SEM_CUDA(w->scales.ensure((size_t)n_out * (k_in / 32) * 4));
  SEM_CUDA(w->planes.ensure((size_t)2 * k_in * n_out * 2));
  SEM_CUDA(w->rscale.ensure((size_t)n_out * 4));
  SEM_CUDA(w->lanes.ensure((size_t)k_in * n_out));
  DevBuf staging;
  sem_tensor_view t{"weight", kQ8, 2, {(uint64_t)k_in, (uint64_t)n_out, 0, 0}, w_q8,
                    (uint64_t)n_out * (k_in / 32) * 34};
  int rc = upload_q8_proj(ctx, staging, &t, n_out, k_in, w->proj(), 0);
  if (rc) return rc;
  *out = w.release();
  return SEM_OK;
}

int q8_gemm(sem_q8_weight* w, const float* d_a, int32_t M, float* d_c, void* d_codes, uint32_t* d_absmax,
            void* stream) {
  if (!w || !d_a || !d_c || !d_codes || !d_absmax) return set_error(SEM_EINVAL, "null argument");
  if (M < 0) return set_error(SEM_EINVAL, "q8 gemm: negative row count %d", M);
  if (reinterpret_cast<uintptr_t>(d_codes) & 15)
    return set_error(SEM_EINVAL, "q8 gemm: the codes scratch must be 16-byte aligned");
  DeviceGuard dg(w->ctx->device);
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : w->ctx->stream;
  // one scale for the whole activation buffer (QuantizeSymmetricINT8Into, quantize.go:29-69)
  SEM_CUDA(cudaMemsetAsync(d_absmax, 0, 4, st));
  SeqMeta meta{nullptr, nullptr, nullptr, M, 1};
  SEM_CUDA(launch_absmax(d_a, (int64_t)M * w->k_in, d_absmax, st));
  __half* codes = static_cast<__half*>(d_codes);
  SEM_CUDA(launch_quantize(d_a, nullptr, nullptr, w->k_in, meta, d_absmax, codes, st));
  SEM_CUDA(launch_q8_proj(codes, w->proj(), M, w->n_out, w->k_in, d_absmax, nullptr, d_c, kEpiStore, nullptr, nullptr,
                          st));
  return SEM_OK;
}

int q8_matmul_int8(sem_q8_weight* w, const void* d_codes, const uint32_t* d_absmax, int32_t M, float* d_c,
                   void* stream) {
  if (!w || !d_codes || !d_absmax || !d_c) return set_error(SEM_EINVAL, "null argument");
  if (M < 0) return set_error(SEM_EINVAL, "q8 matmul: negative row count %d", M);
  if (reinterpret_cast<uintptr_t>(d_codes) & 15) return set_error(SEM_EINVAL, "q8 matmul: codes must be 16-byte aligned");
  DeviceGuard dg(w->ctx->device);
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : w->ctx->stream;
  SEM_CUDA(launch_q8_proj(static_cast<const __half*>(d_codes), w->proj(), M, w->n_out, w->k_in, d_absmax, nullptr, d_c,
                          kEpiStore, nullptr, nullptr, st));
  return SEM_OK;
}

void prof_mark(sem_model* m, int stage, cudaStream_t st, bool after) {
  if (m->prof_used == m->prof_events.size()) {
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) return;
    m->prof_events.push_back(e);
  }
  if (!after) m->prof_stage.push_back(stage);
  cudaEventRecord(m->prof_events[m->prof_used++], st);
}

int profile_read(sem_model* m, const char** names, float* total_ms, int32_t* launches, int32_t cap, int32_t* n_out) {
  DeviceGuard dg(m->ctx->device);
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  SEM_CUDA(cudaDeviceSynchronize());
  for (size_t i = 0; i + 1 < m->prof_used; i += 2) {
    float ms = 0.0f;
    SEM_CUDA(cudaEventElapsedTime(&ms, m->prof_events[i], m->prof_events[i + 1]));
    int s = m->prof_stage[i / 2];
    m->prof_ms[s] += ms;
    m->prof_n[s] += 1;
  }
  int n = 0;
  for (int s = 0; s < kStages && n < cap; ++s) {
    if (names) names[n] = kStageNames[s];
    if (total_ms) total_ms[n] = (float)m->prof_ms[s];
    if (launches) launches[n] = m->prof_n[s];
    ++n;
  }
  if (n_out) *n_out = n;
  for (int s = 0; s < kStages; ++s) { m->prof_ms[s] = 0; m->prof_n[s] = 0; }
  m->prof_used = 0;
  m->prof_stage.clear();
  return SEM_OK;
}

}  // namespace sem

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
extern "C" {

const char* sem_last_error(void) { return sem::last_error(); }

int sem_device_count(int* out) {
  return sem::guarded([&]() -> int {
    if (!out) return sem::set_error(SEM_EINVAL, "null argument");
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
      *out = 0;
      return sem::set_error(SEM_EDEVICE, "cudaGetDeviceCount: %s", cudaGetErrorString(e));
    }
    *out = n;
    return SEM_OK;
  });
}

int sem_context_create(int device, sem_context** out) {
  return sem::guarded([&]() -> int {
    if (!out) return sem::set_error(SEM_EINVAL, "null argument");
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || device < 0 || device >= n)
      return sem::set_error(SEM_EDEVICE, "no CUDA device %d (%s)", device,
                            e == cudaSuccess ? "out of range" : cudaGetErrorString(e));
    sem::DeviceGuard dg(device);
    std::unique_ptr<sem_context> c(new sem_context());
    c->device = device;
    e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) return sem::set_error(SEM_EDEVICE, "cudaStreamCreate: %s", cudaGetErrorString(e));
    *out = c.release();
    return SEM_OK;
  });
}

int sem_context_destroy(sem_context* ctx) {
  return sem::guarded([&]() -> int {
    if (!ctx) return SEM_OK;
    {
      sem::DeviceGuard dg(ctx->device);
      cudaStreamSynchronize(ctx->stream);
      ctx->scratch.release();
      cudaStreamDestroy(ctx->stream);
    }
    delete ctx;
    return SEM_OK;
  });
}

void* sem_context_stream(sem_context* ctx) { return ctx ? static_cast<void*>(ctx->stream) : nullptr; }

int sem_model_load(sem_context* ctx, const sem_model_config* cfg, const sem_tensor_view* tensors, int32_t n,
                   sem_model** out) {
  return sem::guarded([&]() -> int {
    return sem::model_load(ctx, cfg, tensors, n, out);
  });
}

int sem_model_load_gguf(sem_context* ctx, const char* path, sem_model** out) {
  return sem::guarded([&]() -> int {
    if (!ctx || !path || !out) return sem::set_error(SEM_EINVAL, "null argument");
    sem::GgufFile f;
    int rc = f.open(path);
    if (rc) return rc;
    sem_model_config cfg;
    if ((rc = sem::gguf_config(f, &cfg))) return rc;
    std::vector<sem_tensor_view> views;
    views.reserve(f.tensors.size());
    for (const auto& t : f.tensors) {
      sem_tensor_view v{};
      v.name = t.name.c_str();
      v.dtype = t.dtype;
      v.n_dims = (uint32_t)t.dims.size();
      for (size_t k = 0; k < t.dims.size() && k < 4; ++k) v.dims[k] = t.dims[k];
      v.data = f.tensor_data(t);
      v.nbytes = t.size;
      views.push_back(v);
    }
    return sem::model_load(ctx, &cfg, views.data(), (int32_t)views.size(), out);
  });
}

int sem_model_config_get(const sem_model* m, sem_model_config* out) {
  return sem::guarded([&]() -> int {
    if (!m || !out) return sem::set_error(SEM_EINVAL, "null argument");
    *out = m->cfg;
    return SEM_OK;
  });
}

int sem_model_free(sem_model* m) {
  return sem::guarded([&]() -> int {
    if (!m) return SEM_OK;
    sem::DeviceGuard dg(m->ctx->device);
    cudaStreamSynchronize(m->ctx->stream);
    for (cudaEvent_t e : m->prof_events) cudaEventDestroy(e);
    sem::drop_graphs(m);
    for (auto& sl : m->slots)
      if (sl.done) cudaEventDestroy(sl.done);
    delete m;
    return SEM_OK;
  });
}

int sem_model_profile(sem_model* m, int32_t enable) {
  return sem::guarded([&]() -> int {
    if (!m) return sem::set_error(SEM_EINVAL, "null argument");
    m->prof = enable != 0;
    return SEM_OK;
  });
}

int sem_model_profile_read(sem_model* m, const char** names, float* total_ms, int32_t* launches, int32_t cap,
                           int32_t* n_out) {
  return sem::guarded([&]() -> int {
    if (!m) return sem::set_error(SEM_EINVAL, "null argument");
    return sem::profile_read(m, names, total_ms, launches, cap, n_out);
  });
}

int sem_embed(sem_model* m, const int32_t* ids, const int32_t* offsets, int32_t n, const int32_t* dims, float* out) {
  return sem::guarded([&]() -> int {
    return sem::model_embed(m, ids, offsets, n, dims, out);
  });
}

int sem_embed_submit(sem_model* m, const int32_t* ids, const int32_t* offsets, int32_t n, const int32_t* dims,
                     uint64_t* ticket) {
  return sem::guarded([&]() -> int {
    return sem::model_embed_submit(m, ids, offsets, n, dims, ticket);
  });
}

int sem_embed_wait(sem_model* m, uint64_t ticket, float* out) {
  return sem::guarded([&]() -> int { return sem::model_embed_wait(m, ticket, out); });
}

int sem_embed_device(sem_model* m, const int32_t* d_ids, const int32_t* h_offsets, int32_t n, int32_t dim, float* d_out,
                     void* stream) {
  return sem::guarded([&]() -> int {
    return sem::model_embed_device(m, d_ids, h_offsets, n, dim, d_out, stream);
  });
}

int sem_model_check(sem_model* m) {
  return sem::guarded([&]() -> int { return sem::model_check(m); });
}

int sem_model_set_faithful(sem_model* m, const sem_faithful_config* cfg) {
  return sem::guarded([&]() -> int { return sem::model_set_faithful(m, cfg); });
}

int sem_q8_weight_create(sem_context* ctx, const void* w_q8, int32_t k_in, int32_t n_out, sem_q8_weight** out) {
  return sem::guarded([&]() -> int {
    return sem::q8_weight_create(ctx, w_q8, k_in, n_out, out);
  });
}

int sem_q8_weight_free(sem_q8_weight* w) {
  return sem::guarded([&]() -> int {
    if (!w) return SEM_OK;
    sem::DeviceGuard dg(w->ctx->device);
    cudaStreamSynchronize(w->ctx->stream);
    delete w;
    return SEM_OK;
  });
}

int sem_q8_matmul_int8(sem_q8_weight* w, const void* d_codes, const uint32_t* d_absmax, int32_t m, float* d_c,
                       void* stream) {
  return sem::guarded([&]() -> int {
    return sem::q8_matmul_int8(w, d_codes, d_absmax, m, d_c, stream);
  });
}

int sem_q8_path(int32_t mode) {
  return sem::guarded([&]() -> int { return sem::set_q8_path(mode); });
}

int sem_q8_gemm(sem_q8_weight* w, const float* d_a, int32_t m, float* d_c, void* d_codes, uint32_t* d_absmax,
                void* stream) {
  return sem::guarded([&]() -> int {
    return sem::q8_gemm(w, d_a, m, d_c, d_codes, d_absmax, stream);
  });
}

}  // extern "C"
