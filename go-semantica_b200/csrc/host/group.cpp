// Several GPUs of one host as one embedding engine: the model replicated on
// every device and each request's sequences split across them inside the
// library, the multi-GPU form of embedPrompts, which fans the prompts of one
// request out over goroutines (pkg/ggufembed/api.go:237-295). No collective is
// involved: each device embeds its share with its own weights, on its own host
// thread, and the vectors return in the caller's order.
#include <algorithm>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "gguf.h"
#include "internal.h"

struct sem_group {
  std::vector<sem_context*> ctxs;
  std::vector<sem_model*> models;
  sem_model_config cfg{};
  std::mutex mu;  // one request at a time (each device's context serialises its own calls too)
};

namespace sem {
namespace {

// Sequence indices per device, balanced by token count: longest first to the
// device holding the fewest tokens (ties to the lower device, then the lower
// index), each list ascending. The rule of go-semantica_b200/sharded.py
// split_sequences, so hosts that split themselves get the same partition.
std::vector<std::vector<int>> split_by_tokens(const int32_t* offsets, int B, int n) {
  std::vector<int> order(B);
  for (int i = 0; i < B; ++i) order[i] = i;
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) {
    return offsets[a + 1] - offsets[a] > offsets[b + 1] - offsets[b];
  });
  std::vector<int64_t> load(n, 0);
  std::vector<std::vector<int>> parts(n);
  for (int i : order) {
    int best = 0;
    for (int d = 1; d < n; ++d)
      if (load[d] < load[best]) best = d;
    parts[best].push_back(i);
    load[best] += offsets[i + 1] - offsets[i];
  }
  for (auto& p : parts) std::sort(p.begin(), p.end());
  return parts;
}

void free_group(sem_group* g) {
  if (!g) return;
  for (sem_model* m : g->models)
    if (m) sem_model_free(m);
  for (sem_context* c : g->ctxs)
    if (c) sem_context_destroy(c);
  delete g;
}

int check_devices(const int32_t* devices, int32_t n) {
  if (!devices || n <= 0) return set_error(SEM_EINVAL, "empty device list");
  for (int i = 0; i < n; ++i)
    for (int j = 0; j < i; ++j)
      if (devices[j] == devices[i]) return set_error(SEM_EINVAL, "device %d listed twice", devices[i]);
  return SEM_OK;
}

// Creates the contexts, then loads the model on every device in parallel.
int load_group(const int32_t* devices, int32_t n, const sem_model_config* cfg, const sem_tensor_view* tensors,
               int32_t nt, sem_group** out) {
  if (int rc = check_devices(devices, n)) return rc;
  if (!cfg || !tensors || !out) return set_error(SEM_EINVAL, "null argument");
  std::unique_ptr<sem_group, void (*)(sem_group*)> g(new sem_group(), free_group);
  g->cfg = *cfg;
  for (int i = 0; i < n; ++i) {
    sem_context* c = nullptr;
    int rc = sem_context_create(devices[i], &c);
    if (rc) return rc;
    g->ctxs.push_back(c);
  }
  g->models.assign(n, nullptr);
  std::vector<int> rcs(n, SEM_OK);
  std::vector<std::string> msgs(n);
  std::vector<std::thread> th;
  for (int i = 0; i < n; ++i)
    th.emplace_back([&, i] {
      rcs[i] = sem_model_load(g->ctxs[i], cfg, tensors, nt, &g->models[i]);
      if (rcs[i]) msgs[i] = sem_last_error();
    });
  for (auto& t : th) t.join();
  for (int i = 0; i < n; ++i)
    if (rcs[i]) return set_error(rcs[i], "device %d: %s", devices[i], msgs[i].c_str());
  *out = g.release();
  return SEM_OK;
}

}  // namespace
}  // namespace sem

extern "C" {

int sem_group_load(const int32_t* devices, int32_t n_devices, const sem_model_config* cfg,
                   const sem_tensor_view* tensors, int32_t n_tensors, sem_group** out) {
  return sem::guarded([&]() -> int {
    return sem::load_group(devices, n_devices, cfg, tensors, n_tensors, out);
  });
}

int sem_group_load_gguf(const int32_t* devices, int32_t n_devices, const char* path, sem_group** out) {
  return sem::guarded([&]() -> int {
    if (int rc = sem::check_devices(devices, n_devices)) return rc;
    if (!path) return sem::set_error(SEM_EINVAL, "null argument");
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
    return sem::load_group(devices, n_devices, &cfg, views.data(), (int32_t)views.size(), out);
  });
}

int sem_group_size(const sem_group* g, int32_t* out) {
  return sem::guarded([&]() -> int {
    if (!g || !out) return sem::set_error(SEM_EINVAL, "null argument");
    *out = (int32_t)g->models.size();
    return SEM_OK;
  });
}

int sem_group_config_get(const sem_group* g, sem_model_config* out) {
  return sem::guarded([&]() -> int {
    if (!g || !out) return sem::set_error(SEM_EINVAL, "null argument");
    *out = g->cfg;
    return SEM_OK;
  });
}

int sem_group_set_faithful(sem_group* g, const sem_faithful_config* cfg) {
  return sem::guarded([&]() -> int {
    if (!g) return sem::set_error(SEM_EINVAL, "null argument");
    std::lock_guard<std::mutex> lk(g->mu);
    std::vector<sem_faithful_config> prev;
    for (sem_model* m : g->models) prev.push_back(sem::model_faithful_get(m));
    for (size_t i = 0; i < g->models.size(); ++i) {
      const int rc = sem_model_set_faithful(g->models[i], cfg);
      if (rc) {  // the devices already switched go back: every replica keeps one setting
        const std::string msg = sem_last_error();
        for (size_t j = 0; j < i; ++j) sem_model_set_faithful(g->models[j], &prev[j]);
        return sem::set_error(rc, "device %d: %s", g->ctxs[i]->device, msg.c_str());
      }
    }
    return SEM_OK;
  });
}

int sem_group_embed(sem_group* g, const int32_t* ids, const int32_t* offsets, int32_t B, const int32_t* dims_in,
                    float* out) {
  return sem::guarded([&]() -> int {
    if (!g) return sem::set_error(SEM_EINVAL, "null argument");
    // the request is checked before any device starts
    std::vector<int32_t> dims;
    int64_t out_floats = 0;
    if (int rc = sem::validate_embed_request(g->cfg, ids, offsets, B, dims_in, out, &dims, &out_floats)) return rc;
    if (B == 0) return SEM_OK;
    std::vector<int64_t> out_off(B + 1, 0);
    for (int s = 0; s < B; ++s) out_off[s + 1] = out_off[s] + dims[s];
    std::lock_guard<std::mutex> lk(g->mu);
    const int n = (int)g->models.size();
    const auto parts = sem::split_by_tokens(offsets, B, n);
    struct Share {
      std::vector<int32_t> ids, offsets, dims;
      std::vector<float> out;
      int rc = SEM_OK;
      std::string msg;
    };
    std::vector<Share> sh(n);
    std::vector<std::thread> th;
    for (int d = 0; d < n; ++d) {
      if (parts[d].empty()) continue;
      Share& x = sh[d];
      x.offsets.push_back(0);
      int64_t floats = 0;
      for (int s : parts[d]) {
        x.ids.insert(x.ids.end(), ids + offsets[s], ids + offsets[s + 1]);
        x.offsets.push_back((int32_t)x.ids.size());
        x.dims.push_back(dims[s]);
        floats += dims[s];
      }
      x.out.resize((size_t)floats);
      th.emplace_back([&g, &x, d] {
        x.rc = sem_embed(g->models[d], x.ids.data(), x.offsets.data(), (int32_t)x.dims.size(), x.dims.data(),
                         x.out.data());
        if (x.rc) x.msg = sem_last_error();
      });
    }
    for (auto& t : th) t.join();
    for (int d = 0; d < n; ++d)
      if (sh[d].rc) return sem::set_error(sh[d].rc, "device %d: %s", g->ctxs[d]->device, sh[d].msg.c_str());
    for (int d = 0; d < n; ++d) {
      int64_t o = 0;
      for (size_t k = 0; k < parts[d].size(); ++k) {
        const int s = parts[d][k];
        std::copy(sh[d].out.begin() + o, sh[d].out.begin() + o + dims[s], out + out_off[s]);
        o += dims[s];
      }
    }
    return SEM_OK;
  });
}

int sem_group_free(sem_group* g) {
  return sem::guarded([&]() -> int {
    sem::free_group(g);
    return SEM_OK;
  });
}

}  // extern "C"
