// Calibration observer behind esmcu_observer (observer.cpp).
#pragma once

#include <cstddef>
#include <memory>
#include <random>
#include <string>
#include <thread>
#include <unordered_map>
#include <utility>
#include <vector>

#include "esm_b200.h"

namespace esmb200 {

class Observer {
 public:
  static constexpr size_t kReservoirSize = 65536;  // observer.h:24

  struct Reservoir {
    std::vector<float> samples;  // |values|, reservoir-sampled
    size_t total_seen = 0;
    std::mt19937 rng{0xc1b1ce};  // observer.h:43
    void feed(const float* values, size_t n);
    float percentile(float pctile) const;
  };

  ~Observer();
  // Feeds |values| into the site's reservoir now (caller thread).
  void observe(const std::string& key, const float* values, size_t n);
  // The same on a worker thread; the values are moved in.  At most one call
  // per site may be pending: wait() before observing a site again.
  void observe_async(const std::string& key, std::vector<float>&& values);
  void wait();
  void clear();
  size_t num_sites() const { return sites_.size(); }
  const std::pair<std::string, std::unique_ptr<Reservoir>>& site_at(size_t i) const {
    return sites_[i];
  }
  const Reservoir* find(const std::string& key) const {
    auto it = index_.find(key);
    return it == index_.end() ? nullptr : sites_[it->second].second.get();
  }

 private:
  Reservoir& site(const std::string& key);
  // Sites in the order they were first observed.
  std::vector<std::pair<std::string, std::unique_ptr<Reservoir>>> sites_;
  std::unordered_map<std::string, size_t> index_;
  std::vector<std::thread> pending_;
};

}  // namespace esmb200
