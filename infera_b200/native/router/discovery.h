// Fleet discovery for the native router: the etcd v3 JSON gateway (range
// snapshot, then a streaming watch from the next revision; re-snapshot on
// any break), or a static list of worker records.
#pragma once

#include <atomic>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "router.h"

namespace ib {

// First registration per model fixes its tokenizer canary; a later worker
// whose canary differs is refused (its block hashes could never match).
class CanaryGate {
 public:
  bool admit(const Worker& w, std::string* why);
  void forget_if_absent(const Pool& pool);

 private:
  std::mutex mu_;
  std::map<std::string, std::pair<std::string, std::string>> ref_;  // model -> (canary json, worker)
};

class EtcdDiscovery {
 public:
  EtcdDiscovery(std::string endpoint, std::string prefix, Pool* pool, CanaryGate* gate)
      : endpoint_(std::move(endpoint)), prefix_(std::move(prefix)), pool_(pool), gate_(gate) {}
  ~EtcdDiscovery() { stop(); }
  void start();
  void stop();
  // true once the first snapshot was applied
  bool wait_ready(double timeout_s);
  std::atomic<uint64_t> events{0}, snapshots{0}, rejected{0};

 private:
  void run();
  bool snapshot();
  void watch();
  void apply_put(const std::string& value_b64);
  std::string post(const std::string& path, const std::string& body, int* status);
  std::string endpoint_, prefix_;
  Pool* pool_;
  CanaryGate* gate_;
  std::thread th_;
  std::atomic<bool> stop_{false}, ready_{false};
  int64_t rev_ = 0;
};

// records from a JSON file: a list of registration payloads
bool load_static_workers(const std::string& path, Pool* pool, std::string* err);

}  // namespace ib
