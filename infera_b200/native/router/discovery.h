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

// Kubernetes: Pods matching a label selector that carry the annotation
// infera.amd.com/worker-info (the registration record) are workers; a Pod
// with a deletionTimestamp stays in the pool as draining (in-flight
// streams finish, nothing new is routed); DELETED or a missing annotation
// removes it. List, then watch from the list's resourceVersion; any break
// re-lists, which also reconciles deletes the watch missed. The API is
// reached over https (service-account token + CA) or plain http (e.g. a
// `kubectl proxy` sidecar).
struct K8sConfig {
  std::string api_url;       // https://host:port or http://host:port
  std::string namespace_;
  std::string selector;
  std::string token_file;    // bearer token (read at every connect; empty: none)
  std::string ca_file;       // CA bundle for https (empty: system store)
};

class K8sDiscovery {
 public:
  K8sDiscovery(K8sConfig cfg, Pool* pool, CanaryGate* gate) : cfg_(std::move(cfg)), pool_(pool), gate_(gate) {}
  ~K8sDiscovery() { stop(); }
  void start();
  void stop();
  bool wait_ready(double timeout_s);
  std::atomic<uint64_t> events{0}, relists{0}, rejected{0};

 private:
  void run();
  bool relist();
  void watch();
  void handle(const std::string& kind, const Value& pod);
  // GET path on the API server; opens a connection the caller reads from
  struct Stream;
  bool open_get(const std::string& path_query, Stream* st, int* status);
  K8sConfig cfg_;
  Pool* pool_;
  CanaryGate* gate_;
  std::thread th_;
  std::atomic<bool> stop_{false}, ready_{false};
  std::string rv_ = "0";
  std::map<std::string, std::string> pod_worker_;  // pod name -> worker id
};

// records from a JSON file: a list of registration payloads
bool load_static_workers(const std::string& path, Pool* pool, std::string* err);

}  // namespace ib
