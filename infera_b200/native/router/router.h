// Routing core of the native router: worker records and the pool snapshot,
// cache hints, tokenization for block hashing, the KV index fed by engine
// events, the circuit breaker and the routing policies.
//
// Semantics match the Python router (infera_b200/router/*), which follows
// the reference router (infera/router/policy/kv_event_aware.py:33-427,
// infera/router/breaker.py:69-304, infera/router/cache_control.py:67-466,
// infera/router/kv_event/client.py:104-350); the Rust twin of the
// reference (rust/router/src/policy.rs:125-173, pool.rs:77-114) keeps the
// same constants.
#pragma once

#include <atomic>
#include <cstdint>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <shared_mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "json.h"

namespace ib {

uint64_t xxh3_64(const void* p, size_t n);
// h_i = XXH3_64(h_{i-1} as u64 LE || block tokens as u32 LE); full blocks only
std::vector<uint64_t> chain_hashes(const std::vector<uint32_t>& ids, int block_size, uint64_t parent = 0);

// ---------------------------------------------------------------------------
// workers

struct Worker {
  std::string worker_id, url, model_name, engine = "infera-b200", disagg_mode = "mixed";
  std::string status = "active";
  std::string kv_events_endpoint;
  int kv_block_size = 0;
  int dp_rank = -1;  // -1: none
  int dp_size = 0;
  Value record;      // the registration payload as received
  static bool from_json(const Value& v, Worker* w, std::string* err);
  Value to_public() const;
};
using WorkerPtr = std::shared_ptr<const Worker>;
using Snapshot = std::vector<WorkerPtr>;

struct Target {
  WorkerPtr w;
  int dp_rank = -1;
  std::string route_key() const;
};
std::vector<Target> expand_targets(const std::vector<WorkerPtr>& ws);

// Readers take an immutable snapshot with one atomic load; writers rebuild
// it under a mutex (registry callbacks are rare).
class Pool {
 public:
  Pool() : snap_(std::make_shared<const Snapshot>()) {}
  std::shared_ptr<const Snapshot> snapshot() const { return std::atomic_load(&snap_); }
  void upsert(const Worker& w);
  bool remove(const std::string& worker_id);
  std::vector<WorkerPtr> active(const std::string& model, const std::string& mode) const;
  std::vector<std::string> models() const;
  std::function<void(const WorkerPtr&)> on_added;
  std::function<void(const std::string&)> on_removed;

 private:
  std::mutex mu_;
  std::shared_ptr<const Snapshot> snap_;
};

// ---------------------------------------------------------------------------
// cache hints

enum class Retention { None = 0, Short = 1, Long = 2 };
const char* retention_name(Retention r);

struct CacheHints {
  Retention retention = Retention::None;
  std::string session_id;
  bool explicit_hint = false;
  bool multimodal = false;
};
CacheHints parse_cache_hints(const Value& body);
std::vector<uint64_t> image_keys(const Value& body);
Retention effective_retention(Retention r);

// ---------------------------------------------------------------------------
// tokenization for block hashing (the engine's tokenizer, restated)

class Tokenizer {
 public:
  virtual ~Tokenizer() = default;
  virtual std::vector<uint32_t> encode(const std::string& text) const = 0;
  virtual std::vector<uint32_t> chat(const Value& messages) const = 0;
  // false: this text's ids cannot be known exactly (route without locality)
  virtual bool try_encode(const std::string& text, std::vector<uint32_t>* out) const {
    *out = encode(text);
    return true;
  }
  virtual bool try_chat(const Value& messages, std::vector<uint32_t>* out) const {
    *out = chat(messages);
    return true;
  }
};
// UTF-8 bytes at [base, base + 256); base 1000 for vocabularies >= 2048
std::unique_ptr<Tokenizer> make_byte_tokenizer(int vocab_size);
// HF tokenizer.json with a WordLevel model and whitespace pre-tokenization;
// nullptr if the file is another kind
std::unique_ptr<Tokenizer> load_wordlevel_tokenizer(const std::string& path, std::string* err);
// HF tokenizer.json with a byte-level BPE model (GPT-2 / Llama-3 / Qwen2
// families; bpe.cpp lists what is supported); nullptr + err otherwise
std::unique_ptr<Tokenizer> load_bpe_tokenizer(const Value& tokenizer_json, std::string* err);
// WordLevel or byte-level BPE, by the file's model type
std::unique_ptr<Tokenizer> load_tokenizer_json(const std::string& path, std::string* err);
// text of an OpenAI message content: a string, or its text blocks joined
std::string chat_content_text(const Value* content);
// token ids of a completions / chat body; false if they cannot be known
bool request_token_ids(const Value& body, const Tokenizer* tok, std::vector<uint32_t>* out);

// ---------------------------------------------------------------------------
// KV index: the router's view of every worker's prefix cache

class KvIndex {
 public:
  ~KvIndex();
  void add_worker(const WorkerPtr& w);
  void remove_worker(const std::string& worker_id);
  // apply one decoded event batch (vLLM map encoding or SGLang array encoding)
  void apply_batch(const std::string& worker_id, const Value& batch, int rank);
  // length of the run of `hashes` present in the view
  size_t hits(const std::string& worker_id, int rank, const std::vector<uint64_t>& hashes) const;
  size_t view_size(const std::string& worker_id, int rank) const;
  std::vector<uint64_t> view(const std::string& worker_id, int rank, size_t limit) const;
  std::map<std::string, size_t> sizes() const;
  std::atomic<uint64_t> stored{0}, removed{0}, dropped_parent{0}, decode_errors{0}, batches{0};

 private:
  struct RankView {
    std::unordered_set<uint64_t> blocks;
    std::unordered_map<std::string, uint64_t> engine_to_router;
  };
  struct Entry {
    int block_size = 16;
    std::map<int, RankView> ranks;
    std::shared_ptr<std::atomic<bool>> stop;
    std::vector<std::thread> subs;
  };
  void subscribe_loop(std::string worker_id, std::string endpoint, int rank, std::shared_ptr<std::atomic<bool>> stop);
  void apply_event(Entry& e, RankView& rv, const Value& ev);
  mutable std::shared_mutex mu_;
  std::unordered_map<std::string, Entry> workers_;
};

// ---------------------------------------------------------------------------
// circuit breaker

class Breaker {
 public:
  Breaker(int threshold, double cooldown_s, double max_cooldown_s, double probe_timeout_s = 60.0)
      : threshold_(threshold), cooldown_(cooldown_s), max_cooldown_(max_cooldown_s), probe_timeout_(probe_timeout_s) {}
  static bool is_fault(int status) { return status >= 500 || status == 0; }
  bool allows(const std::string& wid);
  std::vector<WorkerPtr> filter(const std::vector<WorkerPtr>& ws);
  void success(const std::string& wid);
  void failure(const std::string& wid, int status);
  void forget(const std::string& wid);
  // 0 closed, 1 half-open, 2 open
  std::map<std::string, std::pair<int, uint64_t>> states();
  std::function<double()> now;

 private:
  struct E {
    int failures = 0;
    int state = 0;  // 0 closed, 1 half-open, 2 open
    double open_until = 0, next_cooldown = 0;
    double probe_at = -1;
    uint64_t trips = 0;
  };
  double t() const;
  std::mutex mu_;
  std::unordered_map<std::string, E> e_;
  int threshold_;
  double cooldown_, max_cooldown_, probe_timeout_;
};

// ---------------------------------------------------------------------------
// policies

struct Pick {
  Target target;
  std::vector<uint64_t> blocks;
  size_t hits = 0;
};

class Policy {
 public:
  virtual ~Policy() = default;
  virtual const char* name() const = 0;
  // role: "mixed", "prefill" or "decode"
  virtual bool pick(const std::vector<WorkerPtr>& cands, const Value& body, const std::vector<uint32_t>* ids,
                    const CacheHints& hints, const std::string& role, Pick* out) = 0;
  virtual void started(const std::string&, const std::vector<uint64_t>&) {}
  virtual void finished(const std::string&, const std::vector<uint64_t>&) {}
  virtual void worker_removed(const std::string&) {}
  virtual size_t active_blocks(const std::string&) { return 0; }
};

class RoundRobinPolicy : public Policy {
 public:
  const char* name() const override { return "round-robin"; }
  bool pick(const std::vector<WorkerPtr>& cands, const Value& body, const std::vector<uint32_t>* ids,
            const CacheHints& hints, const std::string& role, Pick* out) override;

 private:
  std::mutex mu_;
  std::map<std::string, uint64_t> ctr_;
};

class KvAwarePolicy : public Policy {
 public:
  KvAwarePolicy(KvIndex* index, double w, double wp, double wd) : index_(index), w_(w), wp_(wp), wd_(wd) {}
  const char* name() const override { return "kv-aware"; }
  bool pick(const std::vector<WorkerPtr>& cands, const Value& body, const std::vector<uint32_t>* ids,
            const CacheHints& hints, const std::string& role, Pick* out) override;
  void started(const std::string& key, const std::vector<uint64_t>& blocks) override;
  void finished(const std::string& key, const std::vector<uint64_t>& blocks) override;
  void worker_removed(const std::string& wid) override;
  size_t active_blocks(const std::string& key) override;

  static constexpr double kLongAmplifier = 2.0;
  static constexpr double kNoneDampener = 0.1;
  static constexpr size_t kMmAffinityCap = 256;
  static constexpr double kMmBlockWeight = 48.0;
  static constexpr double kRecentDecay = 0.97;
  static constexpr double kUnknownCostBlocks = 1.0;

 private:
  double load_locked(const std::string& key) const;
  KvIndex* index_;
  double w_, wp_, wd_;
  std::mutex mu_;
  std::unordered_map<std::string, std::unordered_map<uint64_t, int>> active_;
  std::unordered_map<std::string, double> recent_;
  std::unordered_map<std::string, std::vector<uint64_t>> mm_;  // LRU, most recent last
};

}  // namespace ib
