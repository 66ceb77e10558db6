// Routing core (see router.h).
#include "router.h"

#define XXH_INLINE_ALL
#include <xxhash.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <sstream>

#include "zmtp.h"

namespace ib {

uint64_t xxh3_64(const void* p, size_t n) { return XXH3_64bits(p, n); }

std::vector<uint64_t> chain_hashes(const std::vector<uint32_t>& ids, int block_size, uint64_t parent) {
  std::vector<uint64_t> out;
  if (block_size <= 0) return out;
  size_t nfull = ids.size() / static_cast<size_t>(block_size);
  out.reserve(nfull);
  std::vector<uint8_t> buf(8 + 4 * static_cast<size_t>(block_size));
  uint64_t h = parent;
  for (size_t b = 0; b < nfull; ++b) {
    for (int k = 0; k < 8; ++k) buf[k] = static_cast<uint8_t>((h >> (8 * k)) & 0xFF);
    const uint32_t* src = ids.data() + b * block_size;
    for (int j = 0; j < block_size; ++j) {
      uint32_t v = src[j];
      uint8_t* d = buf.data() + 8 + 4 * j;
      d[0] = v & 0xFF;
      d[1] = (v >> 8) & 0xFF;
      d[2] = (v >> 16) & 0xFF;
      d[3] = (v >> 24) & 0xFF;
    }
    h = XXH3_64bits(buf.data(), buf.size());
    out.push_back(h);
  }
  return out;
}

// ---------------------------------------------------------------------------
// workers

static std::string str_field(const Value& v, const char* k, const char* dflt = "") {
  const Value* x = v.get(k);
  return x && x->is_str() ? x->s : std::string(dflt);
}

bool Worker::from_json(const Value& v, Worker* w, std::string* err) {
  if (!v.is_obj()) { *err = "record is not an object"; return false; }
  w->worker_id = str_field(v, "worker_id");
  w->url = str_field(v, "url");
  w->model_name = str_field(v, "model_name");
  if (w->worker_id.empty() || w->url.empty() || w->model_name.empty()) {
    *err = "record lacks worker_id / url / model_name";
    return false;
  }
  w->engine = str_field(v, "engine", "infera-b200");
  w->disagg_mode = str_field(v, "disagg_mode", "mixed");
  w->status = str_field(v, "status", "active");
  w->kv_events_endpoint = str_field(v, "kv_events_endpoint");
  const Value* bs = v.get("kv_block_size");
  w->kv_block_size = bs && bs->is_int() ? static_cast<int>(bs->as_int()) : 0;
  if (w->kv_block_size == 0) {
    if (const Value* kv = v.get("kv"))
      if (const Value* ib = kv->get("index_block_size")) w->kv_block_size = static_cast<int>(ib->as_int());
  }
  const Value* r = v.get("dp_rank");
  w->dp_rank = r && r->is_int() ? static_cast<int>(r->as_int()) : -1;
  const Value* s = v.get("dp_size");
  w->dp_size = s && s->is_int() ? static_cast<int>(s->as_int()) : 0;
  w->record = v;
  return true;
}

Value Worker::to_public() const {
  Value v = record.is_obj() ? record : Value::object();
  Value copy = Value::object();
  for (const auto& kv : v.obj()) copy.set(kv.first, kv.second);
  copy.set("status", Value::string(status));
  return copy;
}

std::string Target::route_key() const {
  if (dp_rank < 0 || w->dp_size <= 1 || w->dp_rank >= 0) return w->worker_id;
  return w->worker_id + "#dp" + std::to_string(dp_rank);
}

std::vector<Target> expand_targets(const std::vector<WorkerPtr>& ws) {
  std::vector<Target> out;
  for (const auto& w : ws) {
    if (w->dp_size > 1 && w->dp_rank < 0) {
      for (int r = 0; r < w->dp_size; ++r) out.push_back({w, r});
    } else {
      out.push_back({w, w->dp_rank});
    }
  }
  return out;
}

void Pool::upsert(const Worker& w) {
  WorkerPtr wp = std::make_shared<const Worker>(w);
  bool changed_identity = true;
  {
    std::lock_guard<std::mutex> g(mu_);
    auto cur = std::atomic_load(&snap_);
    auto next = std::make_shared<Snapshot>();
    bool found = false;
    for (const auto& x : *cur) {
      if (x->worker_id == w.worker_id) {
        found = true;
        changed_identity = x->url != w.url || x->kv_events_endpoint != w.kv_events_endpoint ||
                           x->kv_block_size != w.kv_block_size || x->dp_size != w.dp_size;
        next->push_back(wp);
      } else {
        next->push_back(x);
      }
    }
    if (!found) next->push_back(wp);
    std::atomic_store(&snap_, std::shared_ptr<const Snapshot>(std::move(next)));
  }
  if (changed_identity && on_added) on_added(wp);
}

bool Pool::remove(const std::string& worker_id) {
  bool found = false;
  {
    std::lock_guard<std::mutex> g(mu_);
    auto cur = std::atomic_load(&snap_);
    auto next = std::make_shared<Snapshot>();
    for (const auto& x : *cur) {
      if (x->worker_id == worker_id) found = true;
      else next->push_back(x);
    }
    if (found) std::atomic_store(&snap_, std::shared_ptr<const Snapshot>(std::move(next)));
  }
  if (found && on_removed) on_removed(worker_id);
  return found;
}

std::vector<WorkerPtr> Pool::active(const std::string& model, const std::string& mode) const {
  std::vector<WorkerPtr> out;
  auto s = snapshot();
  for (const auto& w : *s) {
    if (w->status != "active") continue;
    if (!model.empty() && w->model_name != model) continue;
    if (!mode.empty() && w->disagg_mode != mode) continue;
    out.push_back(w);
  }
  return out;
}

std::vector<std::string> Pool::models() const {
  std::vector<std::string> out;
  auto s = snapshot();
  for (const auto& w : *s)
    if (w->status == "active" && std::find(out.begin(), out.end(), w->model_name) == out.end())
      out.push_back(w->model_name);
  std::sort(out.begin(), out.end());
  return out;
}

// ---------------------------------------------------------------------------
// cache hints

const char* retention_name(Retention r) {
  return r == Retention::Long ? "long" : r == Retention::Short ? "short" : "none";
}

static std::string trim_lower(const std::string& s) {
  size_t a = 0, b = s.size();
  while (a < b && std::isspace(static_cast<unsigned char>(s[a]))) ++a;
  while (b > a && std::isspace(static_cast<unsigned char>(s[b - 1]))) --b;
  std::string o = s.substr(a, b - a);
  for (auto& c : o) c = static_cast<char>(std::tolower(static_cast<unsigned char>(c)));
  return o;
}

Retention effective_retention(Retention r) {
  if (r != Retention::None) return r;
  const char* e = std::getenv("INFERA_ROUTER_DEFAULT_RETENTION");
  std::string v = e ? trim_lower(e) : "long";
  if (v == "none") return Retention::None;
  if (v == "short") return Retention::Short;
  return Retention::Long;
}

static bool openai_retention(const Value& body, Retention* out) {
  const Value* v = body.get("prompt_cache_retention");
  if (v && v->is_str()) {
    std::string s = trim_lower(v->s);
    if (s == "24h" || s == "1h" || s == "long") { *out = Retention::Long; return true; }
    if (s == "5m" || s == "short") { *out = Retention::Short; return true; }
    if (s == "none" || s == "off" || s == "disabled") { *out = Retention::None; return true; }
    return false;
  }
  const Value* k = body.get("prompt_cache_key");
  if (k && k->truthy()) { *out = Retention::Short; return true; }
  return false;
}

template <typename F>
static void for_cache_control_blocks(const Value& body, F f) {
  if (const Value* sys = body.get("system"); sys && sys->is_arr())
    for (const auto& b : sys->arr())
      if (b.is_obj() && b.get("cache_control")) f(b);
  if (const Value* tools = body.get("tools"); tools && tools->is_arr())
    for (const auto& b : tools->arr())
      if (b.is_obj() && b.get("cache_control")) f(b);
  if (const Value* msgs = body.get("messages"); msgs && msgs->is_arr())
    for (const auto& m : msgs->arr())
      if (const Value* c = m.get("content"); c && c->is_arr())
        for (const auto& b : c->arr())
          if (b.is_obj() && b.get("cache_control")) f(b);
}

template <typename F>
static void for_content_blocks(const Value& body, F f) {
  if (const Value* msgs = body.get("messages"); msgs && msgs->is_arr())
    for (const auto& m : msgs->arr())
      if (const Value* c = m.get("content"); c && c->is_arr())
        for (const auto& b : c->arr())
          if (b.is_obj()) f(b);
  if (const Value* sys = body.get("system"); sys && sys->is_arr())
    for (const auto& b : sys->arr())
      if (b.is_obj()) f(b);
}

static bool block_retention(const Value& b, Retention* out) {
  const Value* t = b.get("type");
  if (t && t->is_str() && (t->s == "thinking" || t->s == "redacted_thinking")) { *out = Retention::None; return true; }
  const Value* cc = b.get("cache_control");
  if (!cc || !cc->is_obj()) return false;
  const Value* ct = cc->get("type");
  if (!ct || !ct->is_str() || ct->s != "ephemeral") return false;
  const Value* ttl = cc->get("ttl");
  if (ttl && ttl->is_str()) {
    std::string s = trim_lower(ttl->s);
    if (s == "1h" || s == "60m" || s == "3600s") { *out = Retention::Long; return true; }
  }
  *out = Retention::Short;
  return true;
}

static bool is_mm_type(const std::string& t) {
  static const char* kinds[] = {"image", "image_url", "input_image", "audio", "input_audio", "video", "video_url",
                                "file", "input_file", "document"};
  for (const char* k : kinds)
    if (t == k) return true;
  return false;
}

CacheHints parse_cache_hints(const Value& body) {
  CacheHints h;
  if (!body.is_obj()) return h;
  Retention oa = Retention::None;
  bool have_oa = openai_retention(body, &oa);
  const Value* sess = body.get("prompt_cache_key");
  if (!sess || !sess->truthy()) sess = body.get("session_id");
  if (sess && sess->is_str()) {
    std::string s = sess->s;
    size_t a = s.find_first_not_of(" \t\n\r"), b = s.find_last_not_of(" \t\n\r");
    if (a != std::string::npos) h.session_id = s.substr(a, b - a + 1);
  }
  bool found = false;
  Retention an = Retention::None;
  for_cache_control_blocks(body, [&](const Value& b) {
    Retention r;
    if (block_retention(b, &r)) {
      if (!found || static_cast<int>(r) > static_cast<int>(an)) an = r;
      found = true;
    }
  });
  bool mm = false;
  for_content_blocks(body, [&](const Value& b) {
    const Value* t = b.get("type");
    if (t && t->is_str() && is_mm_type(t->s)) mm = true;
  });
  if (const Value* im = body.get("images"); im && im->is_arr() && !im->arr().empty()) mm = true;
  if (const Value* au = body.get("audio"); au && (au->is_obj() || au->is_arr()) && au->truthy()) mm = true;
  h.multimodal = mm;
  if (!have_oa && !found) return h;
  Retention best = Retention::None;
  bool any = false;
  if (have_oa) { best = oa; any = true; }
  if (found && (!any || static_cast<int>(an) > static_cast<int>(best))) best = an;
  h.retention = best;
  h.explicit_hint = found || have_oa;
  return h;
}

static const Value* media_ref(const Value& b) {
  if (const Value* iu = b.get("image_url")) {
    if (iu->is_str()) return iu;
    if (const Value* u = iu->get("url"); u && u->is_str()) return u;
  }
  if (const Value* ia = b.get("input_audio"))
    if (const Value* d = ia->get("data"); d && d->is_str()) return d;
  if (const Value* src = b.get("source"))
    for (const char* k : {"url", "data"})
      if (const Value* x = src->get(k); x && x->is_str()) return x;
  for (const char* k : {"url", "data"})
    if (const Value* x = b.get(k); x && x->is_str()) return x;
  return nullptr;
}

std::vector<uint64_t> image_keys(const Value& body) {
  std::vector<uint64_t> keys;
  auto push = [&](const Value* r) {
    if (!r || !r->is_str()) return;
    const std::string& s = r->s;
    size_t a = s.find_first_not_of(" \t\n\r"), b = s.find_last_not_of(" \t\n\r");
    if (a == std::string::npos) return;
    keys.push_back(XXH3_64bits(s.data() + a, b - a + 1));
  };
  if (!body.is_obj()) return keys;
  for_content_blocks(body, [&](const Value& b) { push(media_ref(b)); });
  if (const Value* im = body.get("images"); im && im->is_arr())
    for (const auto& x : im->arr()) push(x.is_str() ? &x : (x.is_obj() ? media_ref(x) : nullptr));
  return keys;
}

// ---------------------------------------------------------------------------
// tokenizers

namespace {

class ByteTok : public Tokenizer {
 public:
  explicit ByteTok(int vocab) {
    base_ = vocab >= 2048 ? 1000 : 0;
    bos_ = vocab > 128010 ? 128000 : vocab - 16;
    start_ = bos_ + 6;
    end_ = bos_ + 9;
  }
  std::vector<uint32_t> encode(const std::string& text) const override {
    std::vector<uint32_t> ids;
    ids.reserve(text.size());
    for (unsigned char c : text) ids.push_back(static_cast<uint32_t>(base_ + c));
    return ids;
  }
  std::vector<uint32_t> chat(const Value& messages) const override {
    std::vector<uint32_t> out{static_cast<uint32_t>(bos_)};
    auto app = [&](const std::string& s) {
      auto e = encode(s);
      out.insert(out.end(), e.begin(), e.end());
    };
    for (const auto& m : messages.arr()) {
      out.push_back(static_cast<uint32_t>(start_));
      const Value* role = m.get("role");
      app((role && role->is_str() ? role->s : std::string(role ? dump_json(*role) : "user")) + "\n");
      app(chat_content_text(m.get("content")));
      out.push_back(static_cast<uint32_t>(end_));
    }
    out.push_back(static_cast<uint32_t>(start_));
    app("assistant\n");
    return out;
  }

 private:
  int base_, bos_, start_, end_;
};

class WordLevelTok : public Tokenizer {
 public:
  std::unordered_map<std::string, uint32_t> vocab;
  uint32_t unk = 0;
  std::vector<uint32_t> encode(const std::string& text) const override {
    std::vector<uint32_t> ids;
    size_t i = 0;
    while (i < text.size()) {
      while (i < text.size() && std::isspace(static_cast<unsigned char>(text[i]))) ++i;
      size_t j = i;
      while (j < text.size() && !std::isspace(static_cast<unsigned char>(text[j]))) ++j;
      if (j > i) {
        auto it = vocab.find(text.substr(i, j - i));
        ids.push_back(it == vocab.end() ? unk : it->second);
      }
      i = j;
    }
    return ids;
  }
  std::vector<uint32_t> chat(const Value& messages) const override {
    std::string text;
    for (const auto& m : messages.arr()) text += chat_content_text(m.get("content")) + " ";
    return encode(text);
  }
};

}  // namespace

std::unique_ptr<Tokenizer> make_byte_tokenizer(int vocab_size) { return std::make_unique<ByteTok>(vocab_size); }

namespace {

std::unique_ptr<Tokenizer> wordlevel_from(const Value& v, std::string* err) {
  const Value* model = v.get("model");
  const Value* type = model ? model->get("type") : nullptr;
  if (!type || !type->is_str() || type->s != "WordLevel") {
    *err = "tokenizer.json is not a WordLevel model";
    return nullptr;
  }
  auto tok = std::make_unique<WordLevelTok>();
  if (const Value* voc = model->get("vocab"))
    for (const auto& kv : voc->obj()) tok->vocab[kv.first] = static_cast<uint32_t>(kv.second.as_int());
  if (const Value* u = model->get("unk_token"); u && u->is_str()) {
    auto it = tok->vocab.find(u->s);
    if (it != tok->vocab.end()) tok->unk = it->second;
  }
  return tok;
}

bool read_json_file(const std::string& path, Value* v, std::string* err) {
  std::ifstream f(path);
  if (!f) {
    *err = "cannot open " + path;
    return false;
  }
  std::stringstream ss;
  ss << f.rdbuf();
  return parse_json(ss.str(), v, err);
}

}  // namespace

std::unique_ptr<Tokenizer> load_wordlevel_tokenizer(const std::string& path, std::string* err) {
  Value v;
  if (!read_json_file(path, &v, err)) return nullptr;
  return wordlevel_from(v, err);
}

std::unique_ptr<Tokenizer> load_tokenizer_json(const std::string& path, std::string* err) {
  Value v;
  if (!read_json_file(path, &v, err)) return nullptr;
  const Value* model = v.get("model");
  const Value* type = model ? model->get("type") : nullptr;
  if (type && type->is_str() && type->s == "BPE") return load_bpe_tokenizer(v, err);
  return wordlevel_from(v, err);
}

bool request_token_ids(const Value& body, const Tokenizer* tok, std::vector<uint32_t>* out) {
  out->clear();
  const Value* prompt = body.get("prompt");
  if (prompt && !prompt->is_null()) {
    if (prompt->is_arr()) {
      const auto& a = prompt->arr();
      if (a.empty() || a[0].is_int()) {
        out->reserve(a.size());
        for (const auto& x : a) out->push_back(static_cast<uint32_t>(x.as_int()));
        return true;
      }
      if (a[0].is_arr()) {
        for (const auto& x : a[0].arr()) out->push_back(static_cast<uint32_t>(x.as_int()));
        return true;
      }
      if (!tok) return false;
      return tok->try_encode(a[0].is_str() ? a[0].s : dump_json(a[0]), out);
    }
    if (!tok) return false;
    return tok->try_encode(prompt->is_str() ? prompt->s : dump_json(*prompt), out);
  }
  if (!tok) return false;
  const Value* msgs = body.get("messages");
  return tok->try_chat(msgs ? *msgs : Value::array(), out);
}

// ---------------------------------------------------------------------------
// KV index

KvIndex::~KvIndex() {
  std::vector<std::thread> all;
  {
    std::unique_lock<std::shared_mutex> g(mu_);
    for (auto& kv : workers_) {
      if (kv.second.stop) kv.second.stop->store(true);
      for (auto& t : kv.second.subs) all.push_back(std::move(t));
    }
    workers_.clear();
  }
  for (auto& t : all)
    if (t.joinable()) t.join();
}

static std::vector<std::pair<int, std::string>> rank_endpoints(const std::string& ep, int dp_size) {
  if (dp_size <= 1) return {{-1, ep}};
  auto colon = ep.rfind(':');
  std::string head = ep.substr(0, colon);
  int port = std::atoi(ep.c_str() + colon + 1);
  std::vector<std::pair<int, std::string>> out;
  for (int r = 0; r < dp_size; ++r) out.emplace_back(r, head + ":" + std::to_string(port + r));
  return out;
}

void KvIndex::add_worker(const WorkerPtr& w) {
  int bs = w->kv_block_size;
  if (bs <= 0) return;
  remove_worker(w->worker_id);
  std::unique_lock<std::shared_mutex> g(mu_);
  Entry& e = workers_[w->worker_id];
  e.block_size = bs;
  e.stop = std::make_shared<std::atomic<bool>>(false);
  if (!w->kv_events_endpoint.empty())
    for (auto& re : rank_endpoints(w->kv_events_endpoint, w->dp_size))
      e.subs.emplace_back(&KvIndex::subscribe_loop, this, w->worker_id, re.second, re.first, e.stop);
}

void KvIndex::remove_worker(const std::string& worker_id) {
  std::vector<std::thread> subs;
  {
    std::unique_lock<std::shared_mutex> g(mu_);
    auto it = workers_.find(worker_id);
    if (it == workers_.end()) return;
    if (it->second.stop) it->second.stop->store(true);
    subs = std::move(it->second.subs);
    workers_.erase(it);
  }
  for (auto& t : subs) t.detach();  // exits within one receive timeout
}

void KvIndex::subscribe_loop(std::string worker_id, std::string endpoint, int rank,
                             std::shared_ptr<std::atomic<bool>> stop) {
  double backoff = 0.25;
  while (!stop->load()) {
    ZmtpSub sub;
    if (!sub.connect(endpoint, "kv-events", 2000)) {
      for (int i = 0; i < static_cast<int>(backoff * 10) && !stop->load(); ++i)
        std::this_thread::sleep_for(std::chrono::milliseconds(100));
      backoff = std::min(backoff * 2, 5.0);
      continue;
    }
    backoff = 0.25;
    std::vector<std::string> frames;
    while (!stop->load()) {
      int r = sub.recv(&frames, 250);
      if (r == 0) continue;
      if (r < 0) break;
      const std::string& payload = frames.back();
      Value batch;
      std::string err;
      if (!parse_msgpack(reinterpret_cast<const uint8_t*>(payload.data()), payload.size(), &batch, &err)) {
        decode_errors++;
        continue;
      }
      if (stop->load()) break;
      apply_batch(worker_id, batch, rank);
    }
  }
}

static std::string hash_key(const Value& h) {
  if (h.is_bin() || h.is_str()) return "b" + h.s;
  uint64_t v = h.as_u64();
  std::string k(9, '\0');
  k[0] = 'i';
  std::memcpy(&k[1], &v, 8);
  return k;
}

void KvIndex::apply_batch(const std::string& worker_id, const Value& batch, int rank) {
  if (!batch.is_arr() || batch.arr().size() < 2) {
    decode_errors++;
    return;
  }
  const auto& a = batch.arr();
  int r = rank;
  if (a.size() >= 3 && a[2].is_int()) r = static_cast<int>(a[2].as_int());
  batches++;
  std::unique_lock<std::shared_mutex> g(mu_);
  auto it = workers_.find(worker_id);
  if (it == workers_.end()) return;
  RankView& rv = it->second.ranks[r];
  for (const auto& ev : a[1].arr()) apply_event(it->second, rv, ev);
}

void KvIndex::apply_event(Entry& e, RankView& rv, const Value& ev) {
  std::string type;
  const Value *hashes = nullptr, *parent = nullptr, *tokens = nullptr, *kind = nullptr;
  if (ev.is_obj()) {
    if (const Value* t = ev.get("type"); t && t->is_str()) type = t->s;
    hashes = ev.get("block_hashes");
    parent = ev.get("parent_block_hash");
    tokens = ev.get("token_ids");
    kind = ev.get("kv_cache_spec_kind");
  } else if (ev.is_arr() && !ev.arr().empty() && ev.arr()[0].is_str()) {
    const auto& x = ev.arr();
    type = x[0].s;
    if (x.size() > 1) hashes = &x[1];
    if (x.size() > 2) parent = &x[2];
    if (x.size() > 3) tokens = &x[3];
  } else {
    decode_errors++;
    return;
  }
  if (type == "BlockStored") {
    if (kind && kind->is_str() && kind->s != "full_attention" && kind->s != "mla_attention" &&
        kind->s != "sink_full_attention")
      return;
    uint64_t p = 0;
    if (parent && !parent->is_null()) {
      auto pit = rv.engine_to_router.find(hash_key(*parent));
      if (pit == rv.engine_to_router.end()) {
        dropped_parent++;
        return;
      }
      p = pit->second;
    }
    std::vector<uint32_t> ids;
    if (tokens)
      for (const auto& t : tokens->arr()) ids.push_back(static_cast<uint32_t>(t.as_int()));
    auto rhs = chain_hashes(ids, e.block_size, p);
    for (uint64_t h : rhs) rv.blocks.insert(h);
    stored += rhs.size();
    if (hashes && hashes->arr().size() == rhs.size())
      for (size_t k = 0; k < rhs.size(); ++k) rv.engine_to_router[hash_key(hashes->arr()[k])] = rhs[k];
  } else if (type == "BlockRemoved") {
    if (!hashes) return;
    for (const auto& h : hashes->arr()) {
      auto it = rv.engine_to_router.find(hash_key(h));
      if (it != rv.engine_to_router.end()) {
        rv.blocks.erase(it->second);
        rv.engine_to_router.erase(it);
        removed++;
      }
    }
  } else if (type == "AllBlocksCleared") {
    rv.blocks.clear();
    rv.engine_to_router.clear();
  }
}

size_t KvIndex::hits(const std::string& worker_id, int rank, const std::vector<uint64_t>& hashes) const {
  if (hashes.empty()) return 0;
  std::shared_lock<std::shared_mutex> g(mu_);
  auto it = workers_.find(worker_id);
  if (it == workers_.end()) return 0;
  auto rit = it->second.ranks.find(rank);
  if (rit == it->second.ranks.end()) return 0;
  size_t n = 0;
  for (uint64_t h : hashes) {
    if (!rit->second.blocks.count(h)) break;
    ++n;
  }
  return n;
}

size_t KvIndex::view_size(const std::string& worker_id, int rank) const {
  std::shared_lock<std::shared_mutex> g(mu_);
  auto it = workers_.find(worker_id);
  if (it == workers_.end()) return 0;
  auto rit = it->second.ranks.find(rank);
  return rit == it->second.ranks.end() ? 0 : rit->second.blocks.size();
}

std::vector<uint64_t> KvIndex::view(const std::string& worker_id, int rank, size_t limit) const {
  std::vector<uint64_t> out;
  std::shared_lock<std::shared_mutex> g(mu_);
  auto it = workers_.find(worker_id);
  if (it == workers_.end()) return out;
  auto rit = it->second.ranks.find(rank);
  if (rit == it->second.ranks.end()) return out;
  for (uint64_t h : rit->second.blocks) {
    if (out.size() >= limit) break;
    out.push_back(h);
  }
  return out;
}

std::map<std::string, size_t> KvIndex::sizes() const {
  std::map<std::string, size_t> out;
  std::shared_lock<std::shared_mutex> g(mu_);
  for (const auto& kv : workers_) {
    size_t n = 0;
    for (const auto& r : kv.second.ranks) n += r.second.blocks.size();
    out[kv.first] = n;
  }
  return out;
}

// ---------------------------------------------------------------------------
// breaker (closed -> open -> half-open -> closed; one probe at a time)

double Breaker::t() const {
  if (now) return now();
  return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

bool Breaker::allows(const std::string& wid) {
  if (threshold_ <= 0) return true;
  std::lock_guard<std::mutex> g(mu_);
  auto it = e_.find(wid);
  if (it == e_.end() || it->second.state == 0) return true;
  E& e = it->second;
  double tt = t();
  if (e.state == 2) {
    if (tt < e.open_until) return false;
    e.state = 1;
  }
  if (e.probe_at >= 0 && tt - e.probe_at < probe_timeout_) return false;
  e.probe_at = tt;
  return true;
}

std::vector<WorkerPtr> Breaker::filter(const std::vector<WorkerPtr>& ws) {
  if (threshold_ <= 0 || ws.empty()) return ws;
  std::vector<WorkerPtr> ok;
  for (const auto& w : ws)
    if (allows(w->worker_id)) ok.push_back(w);
  return ok.empty() ? ws : ok;  // all open: route somewhere rather than nowhere
}

void Breaker::success(const std::string& wid) {
  if (threshold_ <= 0) return;
  std::lock_guard<std::mutex> g(mu_);
  E& e = e_[wid];
  if (e.next_cooldown == 0) e.next_cooldown = cooldown_;
  e.failures = 0;
  e.probe_at = -1;
  e.next_cooldown = cooldown_;
  e.state = 0;
}

void Breaker::failure(const std::string& wid, int status) {
  if (threshold_ <= 0) return;
  std::lock_guard<std::mutex> g(mu_);
  if (!is_fault(status)) {
    auto it = e_.find(wid);
    if (it != e_.end()) it->second.probe_at = -1;
    return;
  }
  E& e = e_[wid];
  if (e.next_cooldown == 0) e.next_cooldown = cooldown_;
  double tt = t();
  if (e.state == 1 || (e.state == 2 && tt >= e.open_until)) {
    e.next_cooldown = std::min(max_cooldown_, e.next_cooldown * 2);
    e.open_until = tt + e.next_cooldown;
    e.probe_at = -1;
    e.trips++;
    e.state = 2;
    return;
  }
  e.failures++;
  if (e.state == 0 && e.failures >= threshold_) {
    e.open_until = tt + e.next_cooldown;
    e.trips++;
    e.state = 2;
  }
}

void Breaker::forget(const std::string& wid) {
  std::lock_guard<std::mutex> g(mu_);
  e_.erase(wid);
}

std::map<std::string, std::pair<int, uint64_t>> Breaker::states() {
  std::map<std::string, std::pair<int, uint64_t>> out;
  std::lock_guard<std::mutex> g(mu_);
  double tt = t();
  for (const auto& kv : e_) {
    int s = kv.second.state;
    if (s == 2 && tt >= kv.second.open_until) s = 1;
    out[kv.first] = {s, kv.second.trips};
  }
  return out;
}

// ---------------------------------------------------------------------------
// policies

bool RoundRobinPolicy::pick(const std::vector<WorkerPtr>& cands, const Value&, const std::vector<uint32_t>*,
                            const CacheHints&, const std::string& role, Pick* out) {
  auto ts = expand_targets(cands);
  if (ts.empty()) return false;
  std::vector<std::string> keys;
  for (const auto& t : ts) keys.push_back(t.route_key());
  std::sort(keys.begin(), keys.end());
  std::string k = role;
  for (const auto& s : keys) k += "|" + s;
  uint64_t i;
  {
    std::lock_guard<std::mutex> g(mu_);
    i = ctr_[k]++;
  }
  out->target = ts[i % ts.size()];
  out->blocks.clear();
  out->hits = 0;
  return true;
}

double KvAwarePolicy::load_locked(const std::string& key) const {
  double a = 0;
  auto it = active_.find(key);
  if (it != active_.end()) a = static_cast<double>(it->second.size());
  auto r = recent_.find(key);
  return a + (r == recent_.end() ? 0.0 : r->second);
}

bool KvAwarePolicy::pick(const std::vector<WorkerPtr>& cands, const Value& body, const std::vector<uint32_t>* ids,
                         const CacheHints& hints, const std::string& role, Pick* out) {
  auto ts = expand_targets(cands);
  if (ts.empty()) return false;
  // block hashes per distinct block size
  std::map<int, std::vector<uint64_t>> hashes;
  for (const auto& t : ts) {
    int bs = t.w->kv_block_size;
    if (bs > 0 && !hashes.count(bs)) hashes[bs] = ids ? chain_hashes(*ids, bs) : std::vector<uint64_t>{};
  }
  double w = role == "prefill" ? wp_ : role == "decode" ? wd_ : w_;
  double amp = w;
  if (hints.retention == Retention::Long) amp *= kLongAmplifier;
  else if (hints.retention == Retention::None && hints.explicit_hint) amp *= kNoneDampener;
  double w_overlap = amp;
  std::vector<uint64_t> mm;
  if (hints.multimodal) {
    w_overlap = 0.0;
    mm = image_keys(body);
  }
  double w_mm = amp * kMmBlockWeight;
  static const std::vector<uint64_t> kEmpty;
  std::lock_guard<std::mutex> g(mu_);
  int best = -1;
  double best_c = 0, best_ld = 0;
  size_t best_hits = 0;
  for (size_t i = 0; i < ts.size(); ++i) {
    const auto& t = ts[i];
    const auto& hs = t.w->kv_block_size > 0 ? hashes[t.w->kv_block_size] : kEmpty;
    size_t hits = index_->hits(t.w->worker_id, t.dp_rank, hs);
    std::string key = t.route_key();
    double ld = load_locked(key);
    size_t mm_hits = 0;
    if (!mm.empty()) {
      auto it = mm_.find(key);
      if (it != mm_.end())
        for (uint64_t k : mm)
          if (std::find(it->second.begin(), it->second.end(), k) != it->second.end()) ++mm_hits;
    }
    double c = w_overlap * static_cast<double>(hs.size() - hits) + w_mm * static_cast<double>(mm.size() - mm_hits) + ld;
    if (best < 0 || c < best_c || (c == best_c && ld < best_ld)) {
      best = static_cast<int>(i);
      best_c = c;
      best_ld = ld;
      best_hits = hits;
    }
  }
  const Target& pk = ts[best];
  std::string key = pk.route_key();
  const auto& hs = pk.w->kv_block_size > 0 ? hashes[pk.w->kv_block_size] : kEmpty;
  // image affinity LRU
  if (!mm.empty()) {
    auto& lru = mm_[key];
    for (uint64_t k : mm) {
      auto it = std::find(lru.begin(), lru.end(), k);
      if (it != lru.end()) lru.erase(it);
      lru.push_back(k);
    }
    while (lru.size() > kMmAffinityCap) lru.erase(lru.begin());
  }
  // recent: decay everyone, charge the pick with the blocks it missed
  for (auto it = recent_.begin(); it != recent_.end();) {
    it->second *= kRecentDecay;
    if (it->second < 1e-3) it = recent_.erase(it);
    else ++it;
  }
  double charge = hs.empty() ? kUnknownCostBlocks : static_cast<double>(hs.size() - best_hits);
  if (charge > 0) recent_[key] += charge;
  out->target = pk;
  out->blocks = hs;
  out->hits = best_hits;
  return true;
}

void KvAwarePolicy::started(const std::string& key, const std::vector<uint64_t>& blocks) {
  if (blocks.empty()) return;
  std::lock_guard<std::mutex> g(mu_);
  auto& refs = active_[key];
  for (uint64_t h : blocks) refs[h]++;
}

void KvAwarePolicy::finished(const std::string& key, const std::vector<uint64_t>& blocks) {
  if (blocks.empty()) return;
  std::lock_guard<std::mutex> g(mu_);
  auto it = active_.find(key);
  if (it == active_.end()) return;
  for (uint64_t h : blocks) {
    auto r = it->second.find(h);
    if (r == it->second.end()) continue;
    if (--r->second <= 0) it->second.erase(r);
  }
}

void KvAwarePolicy::worker_removed(const std::string& wid) {
  std::lock_guard<std::mutex> g(mu_);
  std::string pre = wid + "#dp";
  auto match = [&](const std::string& k) { return k == wid || k.compare(0, pre.size(), pre) == 0; };
  for (auto it = active_.begin(); it != active_.end();) it = match(it->first) ? active_.erase(it) : std::next(it);
  for (auto it = recent_.begin(); it != recent_.end();) it = match(it->first) ? recent_.erase(it) : std::next(it);
  for (auto it = mm_.begin(); it != mm_.end();) it = match(it->first) ? mm_.erase(it) : std::next(it);
}

size_t KvAwarePolicy::active_blocks(const std::string& key) {
  std::lock_guard<std::mutex> g(mu_);
  auto it = active_.find(key);
  return it == active_.end() ? 0 : it->second.size();
}

}  // namespace ib
