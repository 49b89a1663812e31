// Calibration observer: the reference's ActivationObserver
// (observer.h:14-44, observer.cpp:8-51) as a C-ABI object.
//
// Each site keeps a reservoir of at most 65536 |values|, filled by
// Algorithm R with its own std::mt19937 seeded 0xc1b1ce and a fresh
// std::uniform_int_distribution<std::size_t>(0, total_seen) per value past the
// first 65536: the kept positions depend only on that engine's output, so the
// same values fed in the same order keep the same sample as the reference,
// bit for bit (both use the C++ standard library's engine and distribution).
// Percentile(p) sorts a site's sample and takes element
// floor(clamp(p / 100, 0, 1) * float(size - 1)), as the reference indexes it.
//
// The forward feeds every site's tensor in packed row-major order, which is
// the concatenation of the sequences' own [L, d] tensors: one packed forward
// over a calibration set observes the same stream of values as the
// reference's one ForwardWithObserver call per sequence, in that order.
// Feeding runs on worker threads, one site per thread, while the forward
// goes on; esmcu_observer_wait (called at the end of every observed forward)
// joins them, so one site is never fed by two calls at once.
#include "observer.h"

#include <algorithm>
#include <cmath>
#include <cstring>

#include "context.h"

using namespace esmb200;

namespace esmb200 {

void Observer::Reservoir::feed(const float* values, size_t n) {
  for (size_t i = 0; i < n; ++i) {
    const float a = std::fabs(values[i]);
    if (samples.size() < kReservoirSize) {
      samples.push_back(a);
    } else {
      std::uniform_int_distribution<std::size_t> pick(0, total_seen);
      const std::size_t j = pick(rng);
      if (j < kReservoirSize) samples[j] = a;
    }
    ++total_seen;
  }
}

float Observer::Reservoir::percentile(float pctile) const {
  if (samples.empty()) return 0.0f;
  std::vector<float> s = samples;
  const float frac = std::clamp(pctile / 100.0f, 0.0f, 1.0f);
  size_t idx = static_cast<size_t>(std::floor(frac * static_cast<float>(s.size() - 1)));
  if (idx >= s.size()) idx = s.size() - 1;
  std::nth_element(s.begin(), s.begin() + static_cast<long>(idx), s.end());
  return s[idx];
}

Observer::Reservoir& Observer::site(const std::string& key) {
  auto it = index_.find(key);
  if (it != index_.end()) return *sites_[it->second].second;
  index_.emplace(key, sites_.size());
  sites_.emplace_back(key, std::make_unique<Reservoir>());
  return *sites_.back().second;
}

void Observer::observe(const std::string& key, const float* values, size_t n) {
  if (n == 0) return;  // observer.cpp:10: an empty tensor creates no site
  site(key).feed(values, n);
}

void Observer::observe_async(const std::string& key, std::vector<float>&& values) {
  if (values.empty()) return;
  Reservoir* r = &site(key);
  const size_t cap = std::max(1u, std::thread::hardware_concurrency());
  if (pending_.size() >= cap) {
    pending_.front().join();
    pending_.erase(pending_.begin());
  }
  pending_.emplace_back([r, v = std::move(values)]() { r->feed(v.data(), v.size()); });
}

void Observer::wait() {
  for (auto& t : pending_) t.join();
  pending_.clear();
}

void Observer::clear() {
  wait();
  sites_.clear();
  index_.clear();
}

Observer::~Observer() { wait(); }

}  // namespace esmb200

extern "C" {

int esmcu_observer_create(esmcu_observer** out) {
  if (out == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "out is null");
  *out = reinterpret_cast<esmcu_observer*>(new Observer());
  return ESMCU_OK;
}

int esmcu_observer_destroy(esmcu_observer* obs) {
  delete reinterpret_cast<Observer*>(obs);
  return ESMCU_OK;
}

int esmcu_observer_clear(esmcu_observer* obs) {
  if (obs == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "null observer");
  reinterpret_cast<Observer*>(obs)->clear();
  return ESMCU_OK;
}

int esmcu_observer_observe(esmcu_observer* obs, const char* site_key, const float* values,
                           size_t n) {
  if (obs == nullptr || site_key == nullptr)
    return fail(ESMCU_ERR_INVALID_ARGUMENT, "null observer or site key");
  if (n > 0 && values == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "values is null");
  auto* o = reinterpret_cast<Observer*>(obs);
  o->wait();
  o->observe(site_key, values, n);
  return ESMCU_OK;
}

int esmcu_observer_num_sites(const esmcu_observer* obs) {
  if (obs == nullptr) return -1;
  return static_cast<int>(reinterpret_cast<const Observer*>(obs)->num_sites());
}

int esmcu_observer_site(esmcu_observer* obs, int i, float pctile, const char** key,
                        float* value, size_t* total_seen) {
  if (obs == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "null observer");
  auto* o = reinterpret_cast<Observer*>(obs);
  o->wait();
  if (i < 0 || static_cast<size_t>(i) >= o->num_sites())
    return fail(ESMCU_ERR_OUT_OF_RANGE, "site index " + std::to_string(i) + " out of range");
  const auto& s = o->site_at(static_cast<size_t>(i));
  if (key) *key = s.first.c_str();
  if (value) *value = s.second->percentile(pctile);
  if (total_seen) *total_seen = s.second->total_seen;
  return ESMCU_OK;
}

int esmcu_observer_percentile(esmcu_observer* obs, const char* site_key, float pctile,
                              float* value) {
  if (obs == nullptr || site_key == nullptr || value == nullptr)
    return fail(ESMCU_ERR_INVALID_ARGUMENT, "null argument");
  auto* o = reinterpret_cast<Observer*>(obs);
  o->wait();
  const Observer::Reservoir* r = o->find(site_key);
  if (r == nullptr) return fail(ESMCU_ERR_NOT_FOUND, std::string("no site ") + site_key);
  *value = r->percentile(pctile);
  return ESMCU_OK;
}

}  // extern "C"
