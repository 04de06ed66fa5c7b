// Per-op-type device time, the counterpart of the reference's
// ExecutionProfile (lib/src/onnx_graph.dart:22-47): call counts and
// cumulative time per op type, reported sorted by time.  The reference
// times each node with a Stopwatch around _dispatch (:773, :796-802); here
// the work of a call runs on the GPU asynchronously, so every profiled call
// records a CUDA event pair on the session stream around its launches and
// the pairs are read when the report is asked for.
//
// Profiling is off unless enabled.  The events between two kernels end
// their programmatic overlap, so a profiled sequence runs somewhat slower
// than an unprofiled one; calls made while a CUDA graph is being captured
// are not recorded.
#include <algorithm>
#include <cstring>
#include <string>
#include <utility>
#include <vector>

#include "common.cuh"

struct ort_cuda_profile {
  struct Pending {
    std::string op;
    cudaEvent_t e0, e1;
  };
  std::vector<Pending> pending;
  std::vector<cudaEvent_t> spare;
  std::vector<std::string> order;  // op types in first-seen order
  std::unordered_map<std::string, std::pair<int64_t, double>> totals;  // calls, us
};

namespace ortc {
namespace {

cudaEvent_t take_event(ort_cuda_profile* p) {
  if (!p->spare.empty()) {
    cudaEvent_t e = p->spare.back();
    p->spare.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return e;
}

// Folds every completed pair into the totals (the stream has been synchronised).
int fold(ort_cuda_session* s) {
  ort_cuda_profile* p = s->prof;
  for (auto& q : p->pending) {
    float ms = 0.f;
    ORTC_CUDA(cudaEventElapsedTime(&ms, q.e0, q.e1));
    auto it = p->totals.find(q.op);
    if (it == p->totals.end()) {
      p->order.push_back(q.op);
      it = p->totals.emplace(q.op, std::make_pair(int64_t(0), 0.0)).first;
    }
    it->second.first += 1;
    it->second.second += 1000.0 * ms;
    p->spare.push_back(q.e0);
    p->spare.push_back(q.e1);
  }
  p->pending.clear();
  return ORT_CUDA_OK;
}

void destroy_all(ort_cuda_profile* p) {
  for (auto& q : p->pending) {
    cudaEventDestroy(q.e0);
    cudaEventDestroy(q.e1);
  }
  for (cudaEvent_t e : p->spare) cudaEventDestroy(e);
  p->pending.clear();
  p->spare.clear();
}

}  // namespace

OpTimer::OpTimer(ort_cuda_session* s, const char* op) {
  if (!s || !s->prof || !s->profiling || s->capturing) return;
  e0_ = take_event(s->prof);
  if (!e0_) return;
  if (cudaEventRecord(e0_, s->stream) != cudaSuccess) {
    cudaGetLastError();
    s->prof->spare.push_back(e0_);
    e0_ = nullptr;
    return;
  }
  s_ = s;
  op_ = op;
}

OpTimer::~OpTimer() {
  if (!s_) return;
  cudaEvent_t e1 = take_event(s_->prof);
  if (!e1 || cudaEventRecord(e1, s_->stream) != cudaSuccess) {
    cudaGetLastError();
    if (e1) s_->prof->spare.push_back(e1);
    s_->prof->spare.push_back(e0_);
    return;
  }
  s_->prof->pending.push_back({op_, e0_, e1});
}

void profile_free(ort_cuda_session* s) {
  if (!s->prof) return;
  destroy_all(s->prof);
  delete s->prof;
  s->prof = nullptr;
}

}  // namespace ortc

using namespace ortc;

extern "C" {

ORT_CUDA_API int ort_cuda_profile_enable(ort_cuda_session* s, int on) {
  ORTC_CHECK(s, ORT_CUDA_ERR_INVALID_ARG, "session is NULL");
  if (on && !s->prof) s->prof = new ort_cuda_profile();
  s->profiling = on != 0;
  return ORT_CUDA_OK;
}

ORT_CUDA_API int ort_cuda_profile_reset(ort_cuda_session* s) {
  ORTC_CHECK(s, ORT_CUDA_ERR_INVALID_ARG, "session is NULL");
  ORTC_CHECK(!s->capturing, ORT_CUDA_ERR_INVALID_ARG, "cannot synchronise during a capture");
  if (!s->prof) return ORT_CUDA_OK;
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != s->device) ORTC_CUDA(cudaSetDevice(s->device));
  int rc = bounded_sync(s);
  for (auto& q : s->prof->pending) {
    s->prof->spare.push_back(q.e0);
    s->prof->spare.push_back(q.e1);
  }
  s->prof->pending.clear();
  s->prof->totals.clear();
  s->prof->order.clear();
  if (prev >= 0 && prev != s->device) cudaSetDevice(prev);
  return rc;
}

ORT_CUDA_API int ort_cuda_profile_read(ort_cuda_session* s, int index, char* op_type,
                                       int op_type_cap, int64_t* calls, double* device_us) {
  ORTC_CHECK(s && index >= 0, ORT_CUDA_ERR_INVALID_ARG, "bad argument");
  ORTC_CHECK(!s->capturing, ORT_CUDA_ERR_INVALID_ARG, "cannot synchronise during a capture");
  if (!s->prof) return fail(ORT_CUDA_ERR_NOT_FOUND, "no profile entry " + std::to_string(index));
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != s->device) ORTC_CUDA(cudaSetDevice(s->device));
  int rc = ORT_CUDA_OK;
  if (!s->prof->pending.empty()) {
    rc = bounded_sync(s);
    if (rc == ORT_CUDA_OK) rc = fold(s);
  }
  if (prev >= 0 && prev != s->device) cudaSetDevice(prev);
  if (rc) return rc;
  // sorted by cumulative device time, longest first (ExecutionProfile.report)
  std::vector<std::string> ops = s->prof->order;
  std::stable_sort(ops.begin(), ops.end(), [&](const std::string& a, const std::string& b) {
    return s->prof->totals[a].second > s->prof->totals[b].second;
  });
  if (index >= (int)ops.size())
    return fail(ORT_CUDA_ERR_NOT_FOUND, "no profile entry " + std::to_string(index));
  const auto& t = s->prof->totals[ops[index]];
  if (op_type && op_type_cap > 0) {
    std::strncpy(op_type, ops[index].c_str(), (size_t)op_type_cap - 1);
    op_type[op_type_cap - 1] = 0;
  }
  if (calls) *calls = t.first;
  if (device_us) *device_us = t.second;
  return ORT_CUDA_OK;
}

}  // extern "C"
