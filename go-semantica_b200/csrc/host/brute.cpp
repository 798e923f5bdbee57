// search/brute on the device: Builder.Build (builder.go:77-127), Index.SearchVector
// (index.go:29-154), Vector (:162-180) and the BRUT v1 Serializer (storage.go:17-153).
#include <cmath>
#include <cstring>
#include <memory>
#include <unordered_map>
#include <vector>

#include "internal.h"

struct sem_index {
  sem_context* ctx = nullptr;
  int32_t dim = 0, quant = 1;
  int64_t count = 0;
  int row_bytes = 0;  // device row stride (16-byte multiple, zero padded)
  sem::DevBuf data;
  std::vector<int32_t> ids;
  std::unordered_map<int32_t, int64_t> id_to_row;
  sem::DevBuf qin, qprep, cand, out, qthr;
  // int16 rows as byte planes (high bytes, then low bytes) for the tensor-core
  // scan, built at the first exact search; query planes per call
  sem::DevBuf planes, qplanes;
};

namespace sem {
namespace {

int elem_size(int quant) { return quant == 0 ? 4 : quant; }
int padded_row_bytes(int dim, int quant) { return ((dim * elem_size(quant) + 15) / 16) * 16; }

int new_index(sem_context* ctx, int32_t dim, int32_t quant, const int32_t* ids, int64_t count,
              std::unique_ptr<sem_index>* out) {
  if (!ctx) return set_error(SEM_EINVAL, "null context");
  if (quant < 0 || quant > 2) return set_error(SEM_EINVAL, "brute: unsupported quantization %d", quant);
  if (dim <= 0 || dim > 65535) return set_error(SEM_EINVAL, "brute: invalid dimension %d", dim);
  if (count <= 0) return set_error(SEM_EINVAL, "brute: no vectors added");
  if (count > 0x7fffffffLL) return set_error(SEM_EINVAL, "brute: too many rows %lld", (long long)count);
  std::unique_ptr<sem_index> x(new sem_index());
  x->ctx = ctx;
  x->dim = dim;
  x->quant = quant;
  x->count = count;
  x->row_bytes = padded_row_bytes(dim, quant);
  x->ids.resize(count);
  x->id_to_row.reserve((size_t)count);
  for (int64_t i = 0; i < count; ++i) {
    int32_t id = ids ? ids[i] : (int32_t)i;
    if (!x->id_to_row.emplace(id, i).second) return set_error(SEM_EINVAL, "brute: duplicate id %d", id);
    x->ids[i] = id;
  }
  cudaError_t e = x->data.ensure((size_t)count * x->row_bytes);
  if (e != cudaSuccess) return set_error(SEM_ENOMEM, "device allocation failed: %s", cudaGetErrorString(e));
  *out = std::move(x);
  return SEM_OK;
}

// Rows per chunk so that chunks x query-blocks covers the GPU a few times.
ScanPlan plan_for(int64_t count, int nq) {
  int64_t qblocks = (nq + 7) / 8;
  int64_t want = (4 * 148 + qblocks - 1) / qblocks;
  int64_t max_chunks = (count + 255) / 256;
  int64_t chunks = want < 1 ? 1 : want;
  if (chunks > max_chunks) chunks = max_chunks;
  if (chunks < 1) chunks = 1;
  int64_t rpc = (count + chunks - 1) / chunks;
  chunks = (count + rpc - 1) / rpc;
  return ScanPlan{(int32_t)chunks, rpc, 0};
}

// Scan + per-index merge into nq x k keys at d_keys (device), on ctx stream.
int search_keys(sem_index* x, const void* d_queries, int nq, int k, int mode, int64_t row_base, uint64_t* d_keys,
                cudaStream_t st) {
  if (mode == SEM_SEARCH_EXACT && x->quant == 0)
    return set_error(SEM_EINVAL, "brute: exact search needs an int8 or int16 index");
  const int plane_bytes = ((x->dim + 15) / 16) * 16;
  if (mode == SEM_SEARCH_EXACT && x->quant == 2 && scan_exact_tc16_supported(x->dim, plane_bytes, k)) {
    // int16 rows: the tensor-core scan on byte planes (exact int32 scores)
    const size_t cplane = (size_t)x->count * plane_bytes, qplane = (size_t)nq * plane_bytes;
    if (!x->planes.p) {
      SEM_CUDA(x->planes.ensure(2 * cplane));
      SEM_CUDA(launch_split_int16(x->data.p, x->count, x->dim, x->row_bytes, plane_bytes, x->planes.p,
                                  x->planes.as<uint8_t>() + cplane, st));
    }
    SEM_CUDA(x->qplanes.ensure(2 * qplane > 0 ? 2 * qplane : 16));
    SEM_CUDA(launch_split_int16(d_queries, nq, x->dim, x->row_bytes, plane_bytes, x->qplanes.p,
                                x->qplanes.as<uint8_t>() + qplane, st));
    const TcScanPlan tp = plan_scan_exact_tc(x->count, nq);
    const size_t need = (size_t)nq * tp.n_parts * k * sizeof(uint64_t);
    SEM_CUDA(x->cand.ensure(need > 0 ? need : 8));
    SEM_CUDA(x->qthr.ensure((size_t)(nq > 0 ? nq : 1) * 4));
    SEM_CUDA(cudaMemsetAsync(x->qthr.p, 0, (size_t)nq * 4, st));
    uint64_t* cand = x->cand.as<uint64_t>();
    cudaError_t e = launch_scan_exact_tc16(x->planes.p, x->planes.as<uint8_t>() + cplane, x->count, plane_bytes,
                                           x->qplanes.p, x->qplanes.as<uint8_t>() + qplane, nq, k, tp, row_base, cand,
                                           x->qthr.as<uint32_t>(), nullptr, st);
    if (e != cudaSuccess) return set_error(SEM_EDEVICE, "scan: %s", cudaGetErrorString(e));
    e = launch_topk_merge(cand, tp.n_parts, k, (int64_t)tp.n_parts * k, nq, k, k, false, 2, nullptr, nullptr, nullptr,
                          d_keys, st);
    if (e != cudaSuccess) return set_error(SEM_EDEVICE, "merge: %s", cudaGetErrorString(e));
    return SEM_OK;
  }
  if (mode == SEM_SEARCH_EXACT && scan_exact_tc_supported(elem_size(x->quant), x->row_bytes, k, x->data.p, d_queries)) {
    // int8 rows: the tensor-core scan (exact int32 scores)
    const TcScanPlan tp = plan_scan_exact_tc(x->count, nq);
    const size_t need = (size_t)nq * tp.n_parts * k * sizeof(uint64_t);
    SEM_CUDA(x->cand.ensure(need > 0 ? need : 8));
    SEM_CUDA(x->qthr.ensure((size_t)(nq > 0 ? nq : 1) * 4));
    SEM_CUDA(cudaMemsetAsync(x->qthr.p, 0, (size_t)nq * 4, st));
    uint64_t* cand = x->cand.as<uint64_t>();
    cudaError_t e = launch_scan_exact_tc(x->data.p, x->count, x->row_bytes, d_queries, nq, k, tp, row_base, cand,
                                         x->qthr.as<uint32_t>(), nullptr, st);
    if (e != cudaSuccess) return set_error(SEM_EDEVICE, "scan: %s", cudaGetErrorString(e));
    e = launch_topk_merge(cand, tp.n_parts, k, (int64_t)tp.n_parts * k, nq, k, k, false, elem_size(x->quant), nullptr,
                          nullptr, nullptr, d_keys, st);
    if (e != cudaSuccess) return set_error(SEM_EDEVICE, "merge: %s", cudaGetErrorString(e));
    return SEM_OK;
  }
  ScanPlan plan = plan_for(x->count, nq);
  plan.row_base = row_base;
  size_t need = (size_t)nq * plan.chunks * k * sizeof(uint64_t);
  SEM_CUDA(x->cand.ensure(need > 0 ? need : 8));
  uint64_t* cand = x->cand.as<uint64_t>();
  cudaError_t e;
  if (mode == SEM_SEARCH_EXACT)
    e = launch_scan_exact(x->data.p, elem_size(x->quant), x->count, x->dim, d_queries, nq, k, plan, cand, st);
  else
    e = launch_scan_float(x->data.p, elem_size(x->quant), x->count, x->dim, static_cast<const float*>(d_queries), nq, k,
                          plan, cand, st);
  if (e != cudaSuccess) return set_error(SEM_EDEVICE, "scan: %s", cudaGetErrorString(e));
  e = launch_topk_merge(cand, plan.chunks, k, (int64_t)plan.chunks * k, nq, k, k, mode != SEM_SEARCH_EXACT,
                        elem_size(x->quant), nullptr, nullptr, nullptr, d_keys, st);
  if (e != cudaSuccess) return set_error(SEM_EDEVICE, "merge: %s", cudaGetErrorString(e));
  return SEM_OK;
}

}  // namespace

int index_build(sem_context* ctx, int32_t dim, int32_t quant, const float* vectors, const int32_t* ids, int64_t count,
                sem_index** out) {
  if (!vectors || !out) return set_error(SEM_EINVAL, "null argument");
  std::unique_ptr<sem_index> x;
  int rc = new_index(ctx, dim, quant, ids, count, &x);
  if (rc) return rc;
  DeviceGuard dg(ctx->device);
  std::lock_guard<std::mutex> lk(ctx->mu);
  // normalise + quantise on the device in chunks of rows
  const int64_t chunk = 1 << 16;
  DevBuf stage;
  SEM_CUDA(stage.ensure((size_t)chunk * dim * 4));
  for (int64_t r0 = 0; r0 < count; r0 += chunk) {
    int64_t n = count - r0 < chunk ? count - r0 : chunk;
    SEM_CUDA(cudaMemcpyAsync(stage.p, vectors + r0 * dim, (size_t)n * dim * 4, cudaMemcpyHostToDevice, ctx->stream));
    SEM_CUDA(launch_normalize_quantize(stage.as<float>(), n, dim, quant, x->row_bytes, true,
                                       x->data.as<uint8_t>() + r0 * x->row_bytes, ctx->stream));
    SEM_CUDA(cudaStreamSynchronize(ctx->stream));
  }
  *out = x.release();
  return SEM_OK;
}

int index_create(sem_context* ctx, int32_t dim, int32_t quant, const void* data, const int32_t* ids, int64_t count,
                 sem_index** out) {
  if (!data || !out) return set_error(SEM_EINVAL, "null argument");
  std::unique_ptr<sem_index> x;
  int rc = new_index(ctx, dim, quant, ids, count, &x);
  if (rc) return rc;
  DeviceGuard dg(ctx->device);
  std::lock_guard<std::mutex> lk(ctx->mu);
  const size_t src_row = (size_t)dim * elem_size(quant);
  SEM_CUDA(cudaMemset2DAsync(x->data.p, x->row_bytes, 0, x->row_bytes, (size_t)count, ctx->stream));
  // host or device source (unified addressing)
  SEM_CUDA(cudaMemcpy2DAsync(x->data.p, x->row_bytes, data, src_row, src_row, (size_t)count, cudaMemcpyDefault,
                             ctx->stream));
  SEM_CUDA(cudaStreamSynchronize(ctx->stream));
  *out = x.release();
  return SEM_OK;
}

int index_search(sem_index* x, const float* queries, int32_t nq, int32_t dim, int32_t k, int32_t mode,
                 int32_t normalize, int32_t* out_ids, float* out_dist, int32_t* out_scores) {
  if (!x) return set_error(SEM_EINVAL, "null index");
  if (k <= 0) return set_error(SEM_EINVAL, "brute: topK must be positive");
  if (dim != x->dim) return set_error(SEM_EINVAL, "brute: query dimension mismatch: got %d want %d", dim, x->dim);
  if (nq < 0 || (nq > 0 && (!queries || !out_ids || !out_dist))) return set_error(SEM_EINVAL, "null argument");
  if (mode != SEM_SEARCH_EXACT && mode != SEM_SEARCH_REFERENCE) return set_error(SEM_EINVAL, "unknown search mode %d", mode);
  if (nq == 0) return SEM_OK;
  int kk = k < x->count ? k : (int)x->count;  // topK = min(topK, count) (index.go:57-59)
  if (kk > 64) return set_error(SEM_EINVAL, "brute: topK %d above the device limit of 64", kk);
  sem_context* ctx = x->ctx;
  DeviceGuard dg(ctx->device);
  std::lock_guard<std::mutex> lk(ctx->mu);
  cudaStream_t st = ctx->stream;
  SEM_CUDA(x->qin.ensure((size_t)nq * dim * 4));
  SEM_CUDA(cudaMemcpyAsync(x->qin.p, queries, (size_t)nq * dim * 4, cudaMemcpyHostToDevice, st));
  const void* dq;
  if (mode == SEM_SEARCH_EXACT) {
    if (x->quant == 0) return set_error(SEM_EINVAL, "brute: exact search needs an int8 or int16 index");
    SEM_CUDA(x->qprep.ensure((size_t)nq * x->row_bytes));
    SEM_CUDA(launch_normalize_quantize(x->qin.as<float>(), nq, dim, x->quant, x->row_bytes, normalize != 0,
                                       x->qprep.p, st));
    dq = x->qprep.p;
  } else if (normalize) {
    SEM_CUDA(x->qprep.ensure((size_t)nq * dim * 4));
    SEM_CUDA(launch_normalize_quantize(x->qin.as<float>(), nq, dim, 0, dim * 4, true, x->qprep.p, st));
    dq = x->qprep.p;
  } else {
    dq = x->qin.p;
  }
  // out buffer: keys (nq*kk u64) then rows, scores (i32), dist (f32)
  size_t keys_b = (size_t)nq * kk * 8;
  SEM_CUDA(x->out.ensure(keys_b + (size_t)nq * kk * 12));
  uint64_t* keys = x->out.as<uint64_t>();
  int32_t* rows = reinterpret_cast<int32_t*>(x->out.as<uint8_t>() + keys_b);
  int32_t* scores = rows + (size_t)nq * kk;
  float* dist = reinterpret_cast<float*>(scores + (size_t)nq * kk);
  int rc = search_keys(x, dq, nq, kk, mode, 0, keys, st);
  if (rc) return rc;
  SEM_CUDA(launch_topk_merge(keys, 1, 0, kk, nq, kk, kk, mode != SEM_SEARCH_EXACT, elem_size(x->quant), rows, scores,
                             dist, nullptr, st));
  std::vector<int32_t> h_rows((size_t)nq * kk), h_scores((size_t)nq * kk);
  std::vector<float> h_dist((size_t)nq * kk);
  SEM_CUDA(cudaMemcpyAsync(h_rows.data(), rows, h_rows.size() * 4, cudaMemcpyDeviceToHost, st));
  SEM_CUDA(cudaMemcpyAsync(h_scores.data(), scores, h_scores.size() * 4, cudaMemcpyDeviceToHost, st));
  SEM_CUDA(cudaMemcpyAsync(h_dist.data(), dist, h_dist.size() * 4, cudaMemcpyDeviceToHost, st));
  SEM_CUDA(cudaStreamSynchronize(st));
  for (int q = 0; q < nq; ++q)
    for (int j = 0; j < k; ++j) {
      size_t o = (size_t)q * k + j;
      if (j < kk) {
        int32_t r = h_rows[(size_t)q * kk + j];
        out_ids[o] = r >= 0 ? x->ids[r] : -1;
        out_dist[o] = h_dist[(size_t)q * kk + j];
        if (out_scores) out_scores[o] = h_scores[(size_t)q * kk + j];
      } else {
        out_ids[o] = -1;
        out_dist[o] = 0.0f;
        if (out_scores) out_scores[o] = 0;
      }
    }
  return SEM_OK;
}

int index_serialize(sem_index* x, void* buf, size_t cap, size_t* written) {
  if (!x || !written) return set_error(SEM_EINVAL, "null argument");
  if (x->dim > 65535 || x->count > 0xffffffffLL) return set_error(SEM_EINVAL, "brute: index too large for BRUT v1");
  const size_t src_row = (size_t)x->dim * elem_size(x->quant);
  const size_t total = 20 + 4 * (size_t)x->count + src_row * (size_t)x->count;
  *written = total;
  if (!buf) return SEM_OK;
  if (cap < total) return set_error(SEM_EINVAL, "buffer of %zu bytes, need %zu", cap, total);
  uint8_t* p = static_cast<uint8_t*>(buf);
  std::memset(p, 0, 20);
  std::memcpy(p, "BRUT", 4);
  uint16_t ver = 1, dim = (uint16_t)x->dim;
  uint32_t cnt = (uint32_t)x->count;
  std::memcpy(p + 4, &ver, 2);
  std::memcpy(p + 6, &dim, 2);
  std::memcpy(p + 8, &cnt, 4);
  p[12] = (uint8_t)x->quant;
  std::memcpy(p + 20, x->ids.data(), 4 * (size_t)x->count);
  DeviceGuard dg(x->ctx->device);
  std::lock_guard<std::mutex> lk(x->ctx->mu);
  SEM_CUDA(cudaMemcpy2D(p + 20 + 4 * (size_t)x->count, src_row, x->data.p, x->row_bytes, src_row, (size_t)x->count,
                        cudaMemcpyDeviceToHost));
  return SEM_OK;
}

int index_deserialize(sem_context* ctx, const void* bytes, size_t n, sem_index** out) {
  if (!ctx || !bytes || !out) return set_error(SEM_EINVAL, "null argument");
  const uint8_t* p = static_cast<const uint8_t*>(bytes);
  if (n < 20) return set_error(SEM_EFORMAT, "unexpected EOF");
  if (std::memcmp(p, "BRUT", 4) != 0)
    return set_error(SEM_EFORMAT, "brute: invalid magic: \"%c%c%c%c\"", p[0], p[1], p[2], p[3]);
  uint16_t ver, dim;
  uint32_t cnt;
  std::memcpy(&ver, p + 4, 2);
  std::memcpy(&dim, p + 6, 2);
  std::memcpy(&cnt, p + 8, 4);
  int quant = p[12];
  if (ver != 1) return set_error(SEM_EFORMAT, "brute: unsupported version %d", ver);
  if (quant > 2) return set_error(SEM_EFORMAT, "brute: unsupported quantization %d", quant);
  const size_t src_row = (size_t)dim * elem_size(quant);
  if (n < 20 + 4 * (size_t)cnt + src_row * cnt) return set_error(SEM_EFORMAT, "unexpected EOF");
  std::vector<int32_t> ids(cnt);
  std::memcpy(ids.data(), p + 20, 4 * (size_t)cnt);
  return index_create(ctx, dim, quant, p + 20 + 4 * (size_t)cnt, ids.data(), cnt, out);
}

int index_vector(sem_index* x, int32_t id, float* out) {
  if (!x || !out) return set_error(SEM_EINVAL, "null argument");
  auto it = x->id_to_row.find(id);
  if (it == x->id_to_row.end()) return set_error(SEM_ENOTFOUND, "brute: id %d not found", id);
  std::vector<uint8_t> row(x->row_bytes);
  DeviceGuard dg(x->ctx->device);
  {
    std::lock_guard<std::mutex> lk(x->ctx->mu);
    SEM_CUDA(cudaMemcpy(row.data(), x->data.as<uint8_t>() + it->second * x->row_bytes, x->row_bytes,
                        cudaMemcpyDeviceToHost));
  }
  // dequantizeInt8 / dequantizeInt16 (quant.go:43-55): float32(v) * float32(1/scale)
  const float s8 = (float)(1.0 / 127.0), s16 = (float)(1.0 / 32767.0);
  for (int i = 0; i < x->dim; ++i) {
    if (x->quant == 0) std::memcpy(&out[i], row.data() + 4 * i, 4);
    else if (x->quant == 1) out[i] = (float)reinterpret_cast<const int8_t*>(row.data())[i] * s8;
    else out[i] = (float)reinterpret_cast<const int16_t*>(row.data())[i] * s16;
  }
  return SEM_OK;
}

}  // namespace sem

extern "C" {

int sem_index_build(sem_context* ctx, int32_t dim, int32_t quant, const float* vectors, const int32_t* ids, int64_t count,
                    sem_index** out) {
  return sem::guarded([&]() -> int {
    return sem::index_build(ctx, dim, quant, vectors, ids, count, out);
  });
}

int sem_index_create(sem_context* ctx, int32_t dim, int32_t quant, const void* data, const int32_t* ids, int64_t count,
                     sem_index** out) {
  return sem::guarded([&]() -> int {
    return sem::index_create(ctx, dim, quant, data, ids, count, out);
  });
}

int sem_index_free(sem_index* x) {
  return sem::guarded([&]() -> int {
    if (!x) return SEM_OK;
    sem::DeviceGuard dg(x->ctx->device);
    cudaStreamSynchronize(x->ctx->stream);
    delete x;
    return SEM_OK;
  });
}

int sem_index_count(const sem_index* x, int64_t* out) {
  return sem::guarded([&]() -> int {
    if (!x || !out) return sem::set_error(SEM_EINVAL, "null argument");
    *out = x->count;
    return SEM_OK;
  });
}

int sem_index_dimension(const sem_index* x, int32_t* out) {
  return sem::guarded([&]() -> int {
    if (!x || !out) return sem::set_error(SEM_EINVAL, "null argument");
    *out = x->dim;
    return SEM_OK;
  });
}

int sem_index_quantization(const sem_index* x, int32_t* out) {
  return sem::guarded([&]() -> int {
    if (!x || !out) return sem::set_error(SEM_EINVAL, "null argument");
    *out = x->quant;
    return SEM_OK;
  });
}

int sem_index_search(sem_index* x, const float* queries, int32_t nq, int32_t dim, int32_t k, int32_t mode,
                     int32_t normalize, int32_t* out_ids, float* out_dist, int32_t* out_scores) {
  return sem::guarded([&]() -> int {
    return sem::index_search(x, queries, nq, dim, k, mode, normalize, out_ids, out_dist, out_scores);
  });
}

int sem_index_search_keys(sem_index* x, const void* d_queries, int32_t nq, int32_t k, int32_t mode, int64_t row_base,
                          uint64_t* d_keys, void* stream) {
  return sem::guarded([&]() -> int {
    if (!x || !d_queries || !d_keys) return sem::set_error(SEM_EINVAL, "null argument");
    if (k <= 0 || k > 64) return sem::set_error(SEM_EINVAL, "brute: topK must be in 1..64 on the device path");
    sem::DeviceGuard dg(x->ctx->device);
    std::lock_guard<std::mutex> lk(x->ctx->mu);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : x->ctx->stream;
    return sem::search_keys(x, d_queries, nq, k, mode, row_base, d_keys, st);
  });
}

int sem_topk_merge(sem_context* ctx, const uint64_t* d_keys, int32_t lists, int32_t nq, int32_t k, int32_t k_out,
                   int32_t mode, int32_t quant, int32_t* d_rows, int32_t* d_scores, float* d_dist, void* stream) {
  return sem::guarded([&]() -> int {
    if (!ctx || !d_keys) return sem::set_error(SEM_EINVAL, "null argument");
    if (k_out <= 0 || k_out > k || k_out > 64) return sem::set_error(SEM_EINVAL, "invalid k_out %d", k_out);
    sem::DeviceGuard dg(ctx->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    // d_keys: lists x nq x k (one list per shard, as an all-gather lays them out)
    cudaError_t e = sem::launch_topk_merge(d_keys, lists, (int64_t)nq * k, k, nq, k, k_out, mode != SEM_SEARCH_EXACT,
                                           quant == 2 ? 2 : 1, d_rows, d_scores, d_dist, nullptr, st);
    if (e != cudaSuccess) return sem::set_error(SEM_EDEVICE, "merge: %s", cudaGetErrorString(e));
    return SEM_OK;
  });
}

int sem_quantize_queries(const float* queries, int32_t nq, int32_t dim, int32_t quant, void* out_codes) {
  return sem::guarded([&]() -> int {
    if (!queries || !out_codes) return sem::set_error(SEM_EINVAL, "null argument");
    if (quant != 1 && quant != 2) return sem::set_error(SEM_EINVAL, "quant must be 1 or 2");
    // quantizeInt8 / quantizeInt16 (quant.go:17-41) of already-normalised values
    for (int64_t i = 0; i < (int64_t)nq * dim; ++i) {
      float v = queries[i];
      if (v > 1.0f) v = 1.0f;
      else if (v < -1.0f) v = -1.0f;
      if (quant == 1) static_cast<int8_t*>(out_codes)[i] = (int8_t)(int32_t)std::round((double)v * 127.0);
      else static_cast<int16_t*>(out_codes)[i] = (int16_t)(int32_t)std::round((double)v * 32767.0);
    }
    return SEM_OK;
  });
}

int sem_index_vector(sem_index* x, int32_t id, float* out) {
  return sem::guarded([&]() -> int { return sem::index_vector(x, id, out); });
}

int sem_index_serialize(sem_index* x, void* buf, size_t cap, size_t* written) {
  return sem::guarded([&]() -> int {
    return sem::index_serialize(x, buf, cap, written);
  });
}

int sem_index_deserialize(sem_context* ctx, const void* bytes, size_t n, sem_index** out) {
  return sem::guarded([&]() -> int {
    return sem::index_deserialize(ctx, bytes, n, out);
  });
}

}  // extern "C"
