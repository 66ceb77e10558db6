// The native router's HTTP front door and data plane.
//
// Threading: one acceptor; one thread per client connection (keep-alive
// requests on it are served in order). A request's upstream leg runs on the
// same thread with blocking sockets, so the streamed relay is a tight
// read -> write loop with no scheduler in between. Shared state is the pool
// snapshot (one atomic load per request), the KV index (reader lock), the
// policy and breaker (short mutexes) and relaxed atomic counters.
//
// Routes and behaviour follow the Python router (infera_b200/server/app.py,
// infera_b200/router/{auto,mixed,disagg,direct}.py), which follows the
// reference (infera/server/app.py:110-619, infera/router/mixed.py:75-523,
// infera/router/disagg.py:66-1055; rust/router/src/handlers.rs:40-120,
// proxy.rs:304-480).
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <signal.h>
#include <sys/socket.h>
#include <unistd.h>

#include <fstream>

#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <random>
#include <thread>

#include "discovery.h"
#include "net.h"
#include "nats.h"
#include "router.h"

namespace ib {

struct Config {
  std::string host = "0.0.0.0";
  int port = 8000;
  std::string discovery = "etcd";
  std::string etcd_endpoint;
  std::string etcd_prefix = "/infera/workers/";
  std::string static_workers;
  std::string policy = "kv-aware";
  std::string router_mode = "auto";
  std::string tokenizer_path;
  double w = 1.0, wp = -1.0, wd = -1.0;
  int max_retries = 1;
  int migration_limit = 0;
  int breaker_threshold = 3;
  double breaker_cooldown = 5.0, breaker_max_cooldown = 60.0;
  int block_size = 16;
  bool verbose = false;
  std::string request_transport = "http";   // "nats": workers registered with request_transport=bus over NATS
  std::string nats_url = "nats://127.0.0.1:4222";
  double nats_idle_timeout = 900.0;
  double nats_max_duration = 0.0;
  K8sConfig k8s;
};

static double now_s() {
  return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

static std::string rand_hex(int nbytes) {
  static thread_local std::mt19937_64 rng(std::random_device{}() ^ static_cast<uint64_t>(now_s() * 1e9));
  std::string s;
  char b[3];
  for (int i = 0; i < nbytes; ++i) {
    std::snprintf(b, sizeof(b), "%02x", static_cast<unsigned>(rng() & 0xFF));
    s += b;
  }
  return s;
}

static std::string err_json(const std::string& msg) {
  std::string o = "{\"error\":";
  json_escape(msg, o);
  o += "}";
  return o;
}

static const char* kDrainingNotice = "infera-worker-draining";

// ---------------------------------------------------------------------------
// upstream connections (keep-alive, per host:port idle lists)

class UpstreamPool {
 public:
  int get(const std::string& host, int port, bool* reused) {
    std::string k = host + ":" + std::to_string(port);
    {
      std::lock_guard<std::mutex> g(mu_);
      auto& v = idle_[k];
      while (!v.empty()) {
        int fd = v.back();
        v.pop_back();
        char c;
        ssize_t r = ::recv(fd, &c, 1, MSG_PEEK | MSG_DONTWAIT);
        if (r == 0 || (r < 0 && errno != EAGAIN && errno != EWOULDBLOCK)) {
          ::close(fd);  // the worker closed it
          continue;
        }
        *reused = true;
        return fd;
      }
    }
    *reused = false;
    return tcp_connect(host, port, 5000);
  }
  void put(const std::string& host, int port, int fd) {
    std::string k = host + ":" + std::to_string(port);
    std::lock_guard<std::mutex> g(mu_);
    auto& v = idle_[k];
    if (v.size() < 256) v.push_back(fd);
    else ::close(fd);
  }

 private:
  std::mutex mu_;
  std::map<std::string, std::vector<int>> idle_;
};

struct Upstream {
  std::string host;
  int port = 0;
  int fd = -1;
  Conn conn;
  HttpResponseHead head;
  std::unique_ptr<BodyReader> body;
  bool reusable = false;
};

// ---------------------------------------------------------------------------

class App {
 public:
  explicit App(Config c)
      : cfg(std::move(c)),
        breaker(cfg.breaker_threshold, cfg.breaker_cooldown, cfg.breaker_max_cooldown) {
    if (cfg.policy == "round-robin") policy = std::make_unique<RoundRobinPolicy>();
    else
      policy = std::make_unique<KvAwarePolicy>(&index, cfg.w, cfg.wp < 0 ? cfg.w : cfg.wp, cfg.wd < 0 ? cfg.w : cfg.wd);
    if (!cfg.tokenizer_path.empty() && cfg.tokenizer_path.size() > 5 &&
        cfg.tokenizer_path.compare(cfg.tokenizer_path.size() - 5, 5, ".json") == 0) {
      std::string err;
      tok = load_tokenizer_json(cfg.tokenizer_path, &err);
      if (!tok) std::fprintf(stderr, "[ib200_router] tokenizer %s: %s; text prompts route without locality\n",
                             cfg.tokenizer_path.c_str(), err.c_str());
    } else {
      tok = make_byte_tokenizer(128256);
    }
    pool.on_added = [this](const WorkerPtr& w) {
      index.add_worker(w);
      log("worker added: " + w->worker_id + " (" + w->disagg_mode + ")");
    };
    pool.on_removed = [this](const std::string& id) {
      index.remove_worker(id);
      policy->worker_removed(id);
      breaker.forget(id);
      log("worker removed: " + id);
    };
  }

  Config cfg;
  Pool pool;
  KvIndex index;
  CanaryGate gate;
  std::unique_ptr<Policy> policy;
  Breaker breaker;
  std::unique_ptr<Tokenizer> tok;
  std::unique_ptr<EtcdDiscovery> disc;
  std::unique_ptr<K8sDiscovery> k8s;
  std::unique_ptr<NatsConn> nats;   // set with --request-transport nats
  double nats_idle = 900.0;
  double nats_max_duration = 0.0;   // 0: no overall limit
  static constexpr size_t kMaxUnaryBody = size_t(64) << 20;
  UpstreamPool ups;

  // metrics
  std::atomic<uint64_t> req_ok{0}, req_err{0}, inflight{0}, failovers{0}, migrations{0};
  std::atomic<uint64_t> dur_us_sum{0}, dur_count{0}, hit_blocks{0}, req_blocks{0};
  std::mutex pick_mu;
  std::map<std::pair<std::string, std::string>, uint64_t> picks;   // (role, route key) -> n
  std::map<std::string, uint64_t> retention_seen;

  void log(const std::string& m) {
    if (cfg.verbose) std::fprintf(stderr, "[ib200_router] %s\n", m.c_str());
  }

  void count_pick(const std::string& role, const Pick& p) {
    std::lock_guard<std::mutex> g(pick_mu);
    picks[{role, p.target.route_key()}]++;
    hit_blocks += p.hits;
    req_blocks += p.blocks.size();
  }

  // ----------------------------------------------------------------- upstream
  bool open(const Worker& w, const std::string& path, const std::string& body,
            const std::vector<std::pair<std::string, std::string>>& hdrs, Upstream* u, std::string* err) {
    Url url;
    if (!parse_url(w.url, &url)) {
      *err = "bad worker url " + w.url;
      return false;
    }
    std::string req = "POST " + url.path + path + " HTTP/1.1\r\nHost: " + url.host + ":" + std::to_string(url.port) +
                      "\r\nContent-Type: application/json\r\nAccept: text/event-stream, application/json\r\n"
                      "Content-Length: " + std::to_string(body.size()) + "\r\n";
    for (const auto& h : hdrs) req += h.first + ": " + h.second + "\r\n";
    req += "\r\n";
    req += body;
    for (int attempt = 0; attempt < 2; ++attempt) {
      bool reused = false;
      int fd = ups.get(url.host, url.port, &reused);
      if (fd < 0) {
        *err = "connect to " + w.url + " failed";
        return false;
      }
      set_timeouts(fd, 600000, 60000);
      u->host = url.host;
      u->port = url.port;
      u->fd = fd;
      u->conn.reset(fd);
      log("upstream " + w.url + path + (reused ? " (reused)" : " (new)"));
      if (write_all(fd, req) && read_response_head(u->conn, &u->head)) {
        log("upstream status " + std::to_string(u->head.status) + " cl=" + std::to_string(u->head.content_length) +
            (u->head.chunked ? " chunked" : ""));
        u->body = std::make_unique<BodyReader>(u->conn, u->head);
        u->reusable = u->head.keep_alive && (u->head.chunked || u->head.content_length >= 0);
        return true;
      }
      ::close(fd);
      u->fd = -1;
      if (!reused) break;  // a fresh connection failed: the worker is down
    }
    *err = "no response from " + w.url;
    return false;
  }

  void release(Upstream* u, bool complete) {
    if (u->fd < 0) return;
    if (complete && u->reusable && u->conn.buffered() == 0) ups.put(u->host, u->port, u->fd);
    else ::close(u->fd);
    u->fd = -1;
  }

  // body sent to a worker: the client's body plus the retention hint
  std::string forward_body(const Value& body, const CacheHints& h, const Worker& w, bool want_ids) {
    Value out = Value::object();
    for (const auto& kv : body.obj())
      if (kv.first.compare(0, 7, "_infera") != 0) out.set(kv.first, kv.second);
    std::string ret = retention_name(effective_retention(h.retention));
    if (w.engine == "sglang") {
      if (!out.get("priority")) out.set("priority", Value::integer(ret == "long" ? 100 : ret == "short" ? 50 : 0));
      out.set("infera_retention", Value::string(ret));
    } else {
      Value ktp = Value::object();
      if (const Value* old = out.get("kv_transfer_params"); old && old->is_obj())
        for (const auto& kv : old->obj()) ktp.set(kv.first, kv.second);
      if (!ktp.get("infera_retention")) ktp.set("infera_retention", Value::string(ret));
      out.set("kv_transfer_params", ktp);
    }
    if (want_ids) out.set("return_token_ids", Value::boolean(true));
    return dump_json(out);
  }

  static std::vector<std::pair<std::string, std::string>> dp_header(const Target& t) {
    if (t.dp_rank >= 0 && t.w->dp_size > 1) return {{"X-Data-Parallel-Rank", std::to_string(t.dp_rank)}};
    return {};
  }

  // ----------------------------------------------------------------- responses
  struct Reply {
    int status = 0;
    std::string body;
  };

  // Attempt one mixed-role worker. Returns 1 (response fully handled and
  // sent to the client), 0 (failed before any byte reached the client:
  // *fail holds the error response, *fail_status the breaker status).
  static std::string bus_token(const std::string& worker_id) {
    std::string t = worker_id;
    for (char& c : t)
      if (c == '.' || c == ':') c = '_';
    return t;
  }

  static bool wants_bus(const Worker& w) {
    const Value* v = w.record.get("request_transport");
    return v != nullptr && v->is_str() && v->str() == "bus";
  }

  // The bus request transport (workers registered with request_transport=bus):
  // admission on infera.admit.<token>, the request on infera.req.<token> with a
  // private reply subject, frames whose rs-type header is data / done / error;
  // after nats_idle seconds without a frame, or nats_max_duration seconds in
  // total, the request is cancelled on infera.cancel.<token> (three times)
  // and answered 504. Each attempt carries its own bus id (the rid header and
  // the cancel payload): the client's X-Infera-Request-Id is only echoed
  // back, so two client requests with one id never collide on a worker.
  // A lost NATS connection answers 503.
  int attempt_bus(int cfd, const Target& t, const std::vector<uint64_t>& blocks, const Value& body,
                  const CacheHints& hints, const std::string& path, bool stream, const std::string& rid, bool keep,
                  Reply* fail, int* fail_status) {
    const Worker& w = *t.w;
    const std::string token = bus_token(w.worker_id);
    if (!nats->alive()) {
      std::fprintf(stderr, "[ib200_router] bus request to %s refused: NATS connection lost\n", w.worker_id.c_str());
      *fail = {503, err_json("NATS connection lost")};
      *fail_status = -1;   // the router's own failure: not counted against the worker by the breaker
      return 0;
    }
    const std::string bus_rid = rand_hex(16);
    const auto t_start = std::chrono::steady_clock::now();
    policy->started(t.route_key(), blocks);
    struct Done {
      App* a; const Target& t; const std::vector<uint64_t>& b;
      ~Done() { a->policy->finished(t.route_key(), b); }
    } done{this, t, blocks};
    NatsMsg m;
    {
      const std::string inbox = "_INBOX." + rand_hex(12);
      int sid = nats->subscribe(inbox);
      nats->publish("infera.admit." + token, inbox, "", {});
      bool ok = false;
      if (nats->next(sid, 2.0, &m)) {
        Value v;
        std::string perr;
        const Value* okv = parse_json(m.data, &v, &perr) ? v.get("ok") : nullptr;
        ok = okv != nullptr && okv->truthy();
      }
      nats->unsubscribe(sid);
      if (!ok) {
        *fail = {429, err_json("worker at its admission limit")};
        *fail_status = 429;
        return 0;
      }
    }
    std::string hdrs = "{}";
    if (t.dp_rank >= 0 && t.w->dp_size > 1) hdrs = "{\"X-Data-Parallel-Rank\":\"" + std::to_string(t.dp_rank) + "\"}";
    const std::string req = "{\"path\":\"" + path + "\",\"body\":" + forward_body(body, hints, w, false) +
                            ",\"headers\":" + hdrs + "}";
    const std::string inbox = "_INBOX." + rand_hex(12);
    int sid = nats->subscribe(inbox);
    nats->publish("infera.req." + token, inbox, req, {{"rid", bus_rid}});
    auto frame = [&](std::string* kind, int* status) -> bool {
      double wait = nats_idle;
      if (nats_max_duration > 0) {
        const double used = std::chrono::duration<double>(std::chrono::steady_clock::now() - t_start).count();
        wait = std::min(wait, std::max(0.0, nats_max_duration - used));
      }
      if (!nats->next(sid, wait, &m)) return false;
      auto k = m.headers.find("rs-type");
      auto st = m.headers.find("rs-status");
      *kind = k == m.headers.end() ? "data" : k->second;
      *status = st == m.headers.end() ? 200 : std::atoi(st->second.c_str());
      return true;
    };
    auto cancel = [&]() {
      for (int i = 0; i < 3; ++i) nats->publish("infera.cancel." + token, "", bus_rid, {});
    };
    std::string kind;
    int status = 0;
    if (!frame(&kind, &status)) {
      cancel();
      nats->unsubscribe(sid);
      *fail = {504, err_json("worker " + w.worker_id + " sent nothing for " + std::to_string(nats_idle) + " s")};
      *fail_status = 0;
      return 0;
    }
    if (kind == "error") {
      nats->unsubscribe(sid);
      *fail = {status ? status : 502, m.data.empty() ? err_json("worker " + w.worker_id + " failed") : m.data};
      *fail_status = status;
      return 0;
    }
    if (!stream) {
      std::string raw;
      while (kind == "data") {
        raw += m.data;
        if (raw.size() > kMaxUnaryBody) {
          kind = "too_big";
          break;
        }
        if (!frame(&kind, &status)) {
          kind = "timeout";
          break;
        }
      }
      nats->unsubscribe(sid);
      if (kind != "done") {
        if (kind == "timeout" || kind == "too_big") cancel();
        if (kind == "too_big") {
          *fail = {502, err_json("worker " + w.worker_id + " response exceeds " + std::to_string(kMaxUnaryBody) +
                                 " bytes")};
          *fail_status = 0;
          return 0;
        }
        *fail = {kind == "timeout" ? 504 : (status ? status : 502), err_json("worker " + w.worker_id + " failed")};
        *fail_status = kind == "timeout" ? 0 : status;
        return 0;
      }
      send_simple(cfd, 200, "application/json", raw, {{"X-Infera-Request-Id", rid}}, keep);
      breaker.success(w.worker_id);
      return 1;
    }
    write_all(cfd, response_head(200, "text/event-stream", -1,
                                 {{"X-Infera-Request-Id", rid}, {"Cache-Control", "no-cache"}}, keep));
    breaker.success(w.worker_id);
    bool broken = false, ended = false;
    while (true) {
      if (kind == "data") {
        if (!m.data.empty() && !send_chunk(cfd, m.data.data(), m.data.size())) {
          broken = true;
          break;
        }
      } else if (kind == "done") {
        ended = true;
        break;
      } else {   // error frame mid-stream (503: the worker is draining)
        std::string what = status == 503 ? "is shutting down" : "failed";
        std::string msg = "data: " + err_json("worker " + w.worker_id + " " + what + " mid-stream") + "\n\n";
        send_chunk(cfd, msg.data(), msg.size());
        if (status != 503) breaker.failure(w.worker_id, 0);
        ended = true;
        break;
      }
      if (!frame(&kind, &status)) {
        cancel();
        std::string msg = "data: " + err_json("worker " + w.worker_id + " timed out mid-stream") + "\n\n";
        send_chunk(cfd, msg.data(), msg.size());
        ended = true;
        break;
      }
    }
    if (broken) cancel();
    nats->unsubscribe(sid);
    if (ended && !broken) send_last_chunk(cfd);
    return 1;
  }

  int attempt(int cfd, const Target& t, const std::vector<uint64_t>& blocks, const Value& body,
              const CacheHints& hints, const std::string& path, bool stream, const std::string& rid, bool keep,
              Reply* fail, int* fail_status) {
    if (nats && wants_bus(*t.w)) return attempt_bus(cfd, t, blocks, body, hints, path, stream, rid, keep, fail,
                                                    fail_status);
    const Worker& w = *t.w;
    std::string fwd = forward_body(body, hints, w, false);
    Upstream u;
    std::string err;
    policy->started(t.route_key(), blocks);
    struct Done {
      App* a; const Target& t; const std::vector<uint64_t>& b;
      ~Done() { a->policy->finished(t.route_key(), b); }
    } done{this, t, blocks};
    if (!open(w, path, fwd, dp_header(t), &u, &err)) {
      *fail = {502, err_json("worker " + w.worker_id + " failed before first token: " + err)};
      *fail_status = 0;
      return 0;
    }
    if (u.head.status >= 400 || !stream) {
      std::string raw;
      while (u.body->next(&raw)) {
      }
      bool complete = u.body->complete();
      release(&u, complete);
      if (u.head.status >= 400 || !complete) {
        int code = u.head.status >= 400 ? u.head.status : 502;
        *fail = {code, raw.empty() ? err_json("worker " + w.worker_id + " failed") : raw};
        *fail_status = u.head.status >= 400 ? u.head.status : 0;
        return 0;
      }
      send_simple(cfd, u.head.status, "application/json", raw, {{"X-Infera-Request-Id", rid}}, keep);
      breaker.success(w.worker_id);
      return 1;
    }
    // streamed: wait for the first complete event before committing
    std::string buf;
    size_t cut = std::string::npos;
    while ((cut = buf.find("\n\n")) == std::string::npos) {
      if (!u.body->next(&buf)) break;
    }
    if (cut == std::string::npos || (buf.find("\"error\"") != std::string::npos && buf.find("\"error\"") < cut)) {
      release(&u, false);
      *fail = {502, err_json("worker " + w.worker_id + " failed before first token")};
      *fail_status = 0;
      return 0;
    }
    write_all(cfd, response_head(200, "text/event-stream", -1,
                                 {{"X-Infera-Request-Id", rid}, {"Cache-Control", "no-cache"}}, keep));
    breaker.success(w.worker_id);
    bool saw_done = false, broken = false, draining = false;
    while (true) {
      size_t last = buf.rfind("\n\n");
      if (last != std::string::npos) {
        size_t n = last + 2;
        std::string ev(buf, 0, n);
        if (ev.find(kDrainingNotice) != std::string::npos && ev.find("\"error\"") != std::string::npos) {
          draining = true;
          // forward what came before the notice
          size_t at = ev.find("data:", 0);
          size_t notice = ev.find(kDrainingNotice);
          size_t start_of_notice = ev.rfind("data:", notice);
          if (start_of_notice != std::string::npos && start_of_notice > at) send_chunk(cfd, ev.data(), start_of_notice);
          break;
        }
        if (ev.find("data: [DONE]") != std::string::npos) saw_done = true;
        if (!send_chunk(cfd, ev.data(), ev.size())) {
          broken = true;  // client went away
          break;
        }
        buf.erase(0, n);
        if (saw_done) break;
      }
      if (!u.body->next(&buf)) break;
    }
    if (saw_done) {
      std::string rest;
      while (u.body->next(&rest)) {
      }
      release(&u, u.body->complete());
    } else {
      release(&u, false);
    }
    if (!saw_done && !broken) {
      std::string what = draining ? "is shutting down" : "failed";
      std::string msg = "data: " + err_json("worker " + w.worker_id + " " + what + " mid-stream") + "\n\n";
      send_chunk(cfd, msg.data(), msg.size());
      if (!draining) breaker.failure(w.worker_id, 0);
    }
    if (!broken) send_last_chunk(cfd);
    return 1;
  }

  void respond(int cfd, const Reply& r, const std::string& rid, bool keep) {
    send_simple(cfd, r.status, "application/json", r.body, {{"X-Infera-Request-Id", rid}}, keep);
  }

  void dispatch_mixed(int cfd, const Value& body, const std::vector<uint32_t>* ids, const CacheHints& hints,
                      const std::string& path, bool stream, const std::string& rid, bool keep, bool* ok) {
    std::string model;
    if (const Value* m = body.get("model"); m && m->is_str()) model = m->s;
    std::vector<std::string> tried;
    Reply last;
    bool have_last = false;
    for (int k = 0; k <= cfg.max_retries; ++k) {
      auto cands0 = pool.active(model, "mixed");
      std::vector<WorkerPtr> cands;
      for (const auto& w : cands0)
        if (std::find(tried.begin(), tried.end(), w->worker_id) == tried.end()) cands.push_back(w);
      cands = breaker.filter(cands);
      if (cands.empty()) break;
      Pick p;
      if (!policy->pick(cands, body, ids, hints, "mixed", &p)) break;
      count_pick("mixed", p);
      tried.push_back(p.target.w->worker_id);
      int fst = 0;
      if (attempt(cfd, p.target, p.blocks, body, hints, path, stream, rid, keep, &last, &fst)) {
        *ok = true;
        return;
      }
      breaker.failure(p.target.w->worker_id, fst);
      have_last = true;
      failovers++;
      log("failover: " + p.target.w->worker_id + " failed before first byte");
    }
    *ok = false;
    if (have_last) respond(cfd, last, rid, keep);
    else respond(cfd, {503, err_json("no active mixed worker for model='" + model + "'")}, rid, keep);
  }

  // ----------------------------------------------------------------- PD
  struct Proto {
    std::string name;
    bool concurrent = true;
  };

  static std::string meta_protocol(const Worker& w) {
    const Value* m = w.record.get("disagg_meta");
    const Value* p = m ? m->get("protocol") : nullptr;
    return p && p->is_str() ? p->s : "";
  }
  static const Value* meta_param(const Worker& w, const char* k) {
    const Value* m = w.record.get("disagg_meta");
    const Value* ps = m ? m->get("params") : nullptr;
    return ps ? ps->get(k) : nullptr;
  }

  static void single_token(Value& b) {
    b.set("max_tokens", Value::integer(1));
    b.set("stream", Value::boolean(false));
    b.erase("stream_options");
    if (b.get("max_completion_tokens")) b.set("max_completion_tokens", Value::integer(1));
  }
  static void remaining(Value& b) {
    for (const char* k : {"max_tokens", "max_completion_tokens"})
      if (const Value* v = b.get(k); v && v->is_int()) b.set(k, Value::integer(std::max<int64_t>(1, v->as_int() - 1)));
  }

  bool shape(const std::string& proto, const Value& base, const Worker& p, const Worker& d, uint64_t room,
             Value* pb, Value* db, std::string* err) {
    *pb = Value::object();
    *db = Value::object();
    for (const auto& kv : base.obj()) { pb->set(kv.first, kv.second); db->set(kv.first, kv.second); }
    if (proto == "b200-nvlink-push") {
      single_token(*pb);
      Value kp = Value::object();
      kp.set("do_remote_decode", Value::boolean(true));
      kp.set("room", Value::uinteger(room));
      kp.set("decode_worker", Value::string(d.worker_id));
      const Value* ep = meta_param(d, "kv_endpoint");
      kp.set("decode_kv_endpoint", ep ? *ep : Value());
      pb->set("kv_transfer_params", kp);
      // the decode instance recomputes the last prompt token and keeps the full token budget
      Value kd = Value::object();
      kd.set("do_remote_prefill", Value::boolean(true));
      kd.set("room", Value::uinteger(room));
      kd.set("prefill_worker", Value::string(p.worker_id));
      db->set("kv_transfer_params", kd);
      return true;
    }
    if (proto == "sglang-bootstrap") {
      const Value* h = meta_param(p, "bootstrap_host");
      const Value* port = meta_param(p, "bootstrap_port");
      if (!h || !port) { *err = "prefill worker lacks bootstrap_host / bootstrap_port"; return false; }
      for (Value* b : {pb, db}) {
        b->set("bootstrap_host", *h);
        b->set("bootstrap_port", Value::integer(port->is_str() ? std::atoll(port->s.c_str()) : port->as_int()));
        b->set("bootstrap_room", Value::uinteger(room));
      }
      return true;
    }
    if (proto == "vllm-mooncake") {
      char xid[48];
      std::snprintf(xid, sizeof(xid), "xfer-%032llx", static_cast<unsigned long long>(room));
      single_token(*pb);
      Value kp = Value::object();
      kp.set("do_remote_decode", Value::boolean(true));
      kp.set("do_remote_prefill", Value::boolean(false));
      kp.set("transfer_id", Value::string(xid));
      pb->set("kv_transfer_params", kp);
      remaining(*db);
      const Value* eid = meta_param(p, "engine_id");
      const Value* addr = meta_param(p, "bootstrap_addr");
      if (!eid || !addr) { *err = "prefill worker lacks engine_id / bootstrap_addr"; return false; }
      std::string engine_id = eid->is_str() ? eid->s : dump_json(*eid);
      if (p.dp_size > 1) engine_id += "_dp" + std::to_string(room % static_cast<uint64_t>(p.dp_size));
      Value kd = Value::object();
      kd.set("do_remote_prefill", Value::boolean(true));
      kd.set("do_remote_decode", Value::boolean(false));
      kd.set("remote_engine_id", Value::string(engine_id));
      kd.set("remote_bootstrap_addr", *addr);
      kd.set("transfer_id", Value::string(xid));
      db->set("kv_transfer_params", kd);
      return true;
    }
    *err = "unknown disagg protocol '" + proto + "'";
    return false;
  }

  void dispatch_pair(int cfd, const Value& body, const CacheHints& hints, const Target& pt,
                     const std::vector<uint64_t>& pblocks, const Target& dt, const std::vector<uint64_t>& dblocks,
                     const std::string& path, bool stream, const std::string& rid, bool keep, bool* ok) {
    const Worker& p = *pt.w;
    const Worker& d = *dt.w;
    std::string pn = meta_protocol(p), dn = meta_protocol(d);
    *ok = false;
    if (pn.empty() || pn != dn) {
      respond(cfd, {500, err_json("protocol mismatch: prefill " + p.worker_id + "='" + pn + "' decode " +
                                  d.worker_id + "='" + dn + "'")}, rid, keep);
      return;
    }
    static thread_local std::mt19937_64 rng(std::random_device{}());
    uint64_t room = rng() >> 1;
    if (pn != "b200-nvlink-push" && pt.dp_rank >= 0 && p.dp_size > 1)
      room = room - room % static_cast<uint64_t>(p.dp_size) + static_cast<uint64_t>(pt.dp_rank);
    Value base = Value::object();
    for (const auto& kv : body.obj())
      if (kv.first.compare(0, 7, "_infera") != 0) base.set(kv.first, kv.second);
    Value pb, db;
    std::string err;
    if (!shape(pn, base, p, d, room, &pb, &db, &err)) {
      respond(cfd, {500, err_json(err)}, rid, keep);
      return;
    }
    db.set("stream", Value::boolean(stream));
    policy->started(pt.route_key(), pblocks);
    policy->started(dt.route_key(), dblocks);
    // prefill leg on its own thread: its KV push must finish even if the client leaves
    std::string pbody = forward_body(pb, hints, p, false);
    auto pstatus = std::make_shared<std::atomic<int>>(-1);
    WorkerPtr pw = pt.w;
    auto phdr = dp_header(pt);
    std::thread prefill([this, pw, path, pbody, phdr, pstatus]() {
      Upstream u;
      std::string e, raw;
      if (!open(*pw, path, pbody, phdr, &u, &e)) {
        pstatus->store(0);
        return;
      }
      while (u.body->next(&raw)) {
      }
      bool complete = u.body->complete();
      release(&u, complete);
      pstatus->store(complete ? u.head.status : 0);
    });
    auto finish = [&]() {
      prefill.join();
      int ps = pstatus->load();
      if (ps >= 200 && ps < 400) breaker.success(p.worker_id);
      else breaker.failure(p.worker_id, ps < 0 ? 0 : ps);
      policy->finished(pt.route_key(), pblocks);
      policy->finished(dt.route_key(), dblocks);
    };
    std::string dbody = forward_body(db, hints, d, false);
    Upstream u;
    bool opened = false;
    int last_status = 502;
    for (int a = 0; a < 3 && !opened; ++a) {
      if (open(d, path, dbody, dp_header(dt), &u, &err) && u.head.status < 400) {
        opened = true;
        break;
      }
      if (u.fd >= 0) {
        last_status = u.head.status;
        release(&u, false);
      }
      std::this_thread::sleep_for(std::chrono::milliseconds(50 << a));
    }
    if (!opened) {
      breaker.failure(d.worker_id, last_status);
      finish();
      respond(cfd, {last_status >= 400 ? last_status : 502, err_json("decode worker " + d.worker_id + " failed to open")},
              rid, keep);
      return;
    }
    breaker.success(d.worker_id);
    if (!stream) {
      std::string raw;
      while (u.body->next(&raw)) {
      }
      release(&u, u.body->complete());
      finish();
      send_simple(cfd, u.head.status, "application/json", raw, {{"X-Infera-Request-Id", rid}}, keep);
      *ok = true;
      return;
    }
    write_all(cfd, response_head(200, "text/event-stream", -1, {{"X-Infera-Request-Id", rid}}, keep));
    std::string buf;
    bool done = false, client_gone = false;
    while (!done) {
      if (!u.body->next(&buf)) break;
      size_t last = buf.rfind("\n\n");
      if (last == std::string::npos) continue;
      if (buf.find("data: [DONE]") != std::string::npos) done = true;
      if (!send_chunk(cfd, buf.data(), last + 2)) {
        client_gone = true;
        break;
      }
      buf.erase(0, last + 2);
    }
    if (done) {
      std::string rest;
      while (u.body->next(&rest)) {
      }
      release(&u, u.body->complete());
    } else {
      release(&u, false);
      if (!client_gone) {
        std::string msg = "data: " + err_json("decode worker " + d.worker_id + " failed mid-stream") + "\n\n";
        send_chunk(cfd, msg.data(), msg.size());
      }
    }
    if (!client_gone) send_last_chunk(cfd);
    finish();
    *ok = true;
  }

  // ----------------------------------------------------------------- front door
  void inference(int cfd, const HttpRequest& req, const std::string& path, bool keep) {
    double t0 = now_s();
    inflight++;
    std::string rid;
    if (const auto* h = req.header("x-infera-request-id")) rid = *h;
    if (rid.empty()) rid = rand_hex(16);
    Value body;
    std::string err;
    bool ok = false;
    if (!parse_json(req.body, &body, &err) || !body.is_obj()) {
      respond(cfd, {400, err_json(body.is_obj() ? "invalid JSON body" : "body must be a JSON object")}, rid, keep);
    } else {
      CacheHints hints = parse_cache_hints(body);
      {
        std::lock_guard<std::mutex> g(pick_mu);
        retention_seen[retention_name(hints.retention)]++;
      }
      std::vector<uint32_t> ids;
      bool have_ids = request_token_ids(body, tok.get(), &ids);
      const std::vector<uint32_t>* idp = have_ids ? &ids : nullptr;
      const Value* sv = body.get("stream");
      bool stream = sv && sv->truthy();
      std::string model;
      if (const Value* m = body.get("model"); m && m->is_str()) model = m->s;
      const std::string* wid = req.header("x-worker-instance-id");
      const std::string* pid = req.header("x-prefill-instance-id");
      if (cfg.router_mode == "direct") {
        direct(cfd, body, hints, wid, pid, path, stream, rid, keep, &ok);
      } else {
        auto ps = pool.active(model, "prefill");
        auto ds = pool.active(model, "decode");
        if (!ps.empty() && !ds.empty()) {
          ps = breaker.filter(ps);
          ds = breaker.filter(ds);
          Pick pp, dp;
          policy->pick(ps, body, idp, hints, "prefill", &pp);
          policy->pick(ds, body, idp, hints, "decode", &dp);
          count_pick("prefill", pp);
          count_pick("decode", dp);
          dispatch_pair(cfd, body, hints, pp.target, pp.blocks, dp.target, dp.blocks, path, stream, rid, keep, &ok);
        } else if ((!ps.empty() || !ds.empty()) && pool.active(model, "mixed").empty()) {
          std::string have = ps.empty() ? "decode" : "prefill", empty = ps.empty() ? "prefill" : "decode";
          respond(cfd, {503, err_json("model '" + model + "' has " + have + " workers but no active " + empty +
                                      " workers")}, rid, keep);
        } else {
          dispatch_mixed(cfd, body, idp, hints, path, stream, rid, keep, &ok);
        }
      }
    }
    (ok ? req_ok : req_err)++;
    inflight--;
    dur_us_sum += static_cast<uint64_t>((now_s() - t0) * 1e6);
    dur_count++;
  }

  void direct(int cfd, const Value& body, const CacheHints& hints, const std::string* wid, const std::string* pid,
              const std::string& path, bool stream, const std::string& rid, bool keep, bool* ok) {
    *ok = false;
    if (!wid || wid->empty()) {
      respond(cfd, {400, err_json("missing x-worker-instance-id header")}, rid, keep);
      return;
    }
    auto find = [&](const std::string& id) -> WorkerPtr {
      auto s = pool.snapshot();
      for (const auto& w : *s)
        if (w->worker_id == id) return w;
      return nullptr;
    };
    WorkerPtr w = find(*wid);
    if (!w) {
      respond(cfd, {404, err_json("unknown worker '" + *wid + "'")}, rid, keep);
      return;
    }
    if (pid && !pid->empty()) {
      WorkerPtr p = find(*pid);
      if (!p) {
        respond(cfd, {404, err_json("unknown prefill worker '" + *pid + "'")}, rid, keep);
        return;
      }
      dispatch_pair(cfd, body, hints, Target{p, p->dp_rank}, {}, Target{w, w->dp_rank}, {}, path, stream, rid, keep, ok);
      return;
    }
    if (w->disagg_mode != "mixed") {
      respond(cfd, {400, err_json("worker '" + *wid + "' is " + w->disagg_mode + "; name a prefill worker too")}, rid,
              keep);
      return;
    }
    Reply fail;
    int fst = 0;
    if (attempt(cfd, Target{w, w->dp_rank}, {}, body, hints, path, stream, rid, keep, &fail, &fst)) {
      *ok = true;
      return;
    }
    breaker.failure(w->worker_id, fst);
    respond(cfd, fail, rid, keep);
  }

  std::string metrics_text() {
    std::string o;
    char b[512];
    auto line = [&](const char* name, const std::string& labels, double v) {
      std::snprintf(b, sizeof(b), "%s{%s} %.17g\n", name, labels.c_str(), v);
      o += b;
    };
    o += "# TYPE infera_requests_total counter\n";
    line("infera_requests_total", "router=\"native\",outcome=\"ok\"", static_cast<double>(req_ok.load()));
    line("infera_requests_total", "router=\"native\",outcome=\"error\"", static_cast<double>(req_err.load()));
    o += "# TYPE infera_requests_inflight gauge\n";
    line("infera_requests_inflight", "router=\"native\"", static_cast<double>(inflight.load()));
    o += "# TYPE infera_request_duration_seconds summary\n";
    line("infera_request_duration_seconds_sum", "router=\"native\"", dur_us_sum.load() / 1e6);
    line("infera_request_duration_seconds_count", "router=\"native\"", static_cast<double>(dur_count.load()));
    o += "# TYPE infera_router_failovers_total counter\n";
    line("infera_router_failovers_total", "router=\"native\"", static_cast<double>(failovers.load()));
    {
      std::lock_guard<std::mutex> g(pick_mu);
      o += "# TYPE infera_router_picks_total counter\n";
      for (const auto& kv : picks)
        line("infera_router_picks_total", "role=\"" + kv.first.first + "\",worker_id=\"" + kv.first.second + "\"",
             static_cast<double>(kv.second));
      o += "# TYPE infera_cache_control_seen_total counter\n";
      for (const auto& kv : retention_seen)
        line("infera_cache_control_seen_total", "retention=\"" + kv.first + "\"", static_cast<double>(kv.second));
    }
    o += "# TYPE infera_router_hit_blocks_total counter\n";
    line("infera_router_hit_blocks_total", "router=\"native\"", static_cast<double>(hit_blocks.load()));
    line("infera_router_request_blocks_total", "router=\"native\"", static_cast<double>(req_blocks.load()));
    auto snap = pool.snapshot();
    std::map<std::string, int> counts;
    for (const auto& w : *snap) counts["model=\"" + w->model_name + "\",mode=\"" + w->disagg_mode + "\",status=\"" +
                                      w->status + "\""]++;
    o += "# TYPE infera_active_workers gauge\n";
    for (const auto& kv : counts) line("infera_active_workers", kv.first, kv.second);
    o += "# TYPE infera_worker_breaker_state gauge\n";
    for (const auto& kv : breaker.states()) {
      line("infera_worker_breaker_state", "worker_id=\"" + kv.first + "\"", kv.second.first);
      line("infera_worker_breaker_trips_total", "worker_id=\"" + kv.first + "\"", static_cast<double>(kv.second.second));
    }
    o += "# TYPE infera_router_cache_view_blocks gauge\n";
    for (const auto& kv : index.sizes())
      line("infera_router_cache_view_blocks", "worker_id=\"" + kv.first + "\"", static_cast<double>(kv.second));
    for (const auto& w : *snap)
      line("infera_policy_active_blocks", "worker_id=\"" + w->worker_id + "\"",
           static_cast<double>(policy->active_blocks(w->worker_id)));
    o += "# TYPE infera_kv_events_total counter\n";
    line("infera_kv_events_total", "kind=\"stored\"", static_cast<double>(index.stored.load()));
    line("infera_kv_events_total", "kind=\"removed\"", static_cast<double>(index.removed.load()));
    line("infera_kv_events_total", "kind=\"dropped_parent\"", static_cast<double>(index.dropped_parent.load()));
    line("infera_kv_events_total", "kind=\"decode_error\"", static_cast<double>(index.decode_errors.load()));
    line("infera_kv_event_batches_total", "router=\"native\"", static_cast<double>(index.batches.load()));
    return o;
  }

  void handle(int cfd, const HttpRequest& req) {
    bool keep = req.keep_alive;
    const std::string& p = req.path;
    if (req.method == "POST" && (p == "/v1/completions" || p == "/v1/chat/completions")) {
      log("request " + p + " bytes=" + std::to_string(req.body.size()));
      inference(cfd, req, p, keep);
      log("request done");
      return;
    }
    if (req.method == "GET" && p == "/health") {
      std::string b = "{\"status\":\"ok\",\"workers\":" + std::to_string(pool.active("", "").size()) +
                      ",\"router\":\"native\"}";
      send_simple(cfd, 200, "application/json", b, {}, keep);
      return;
    }
    if (req.method == "GET" && p == "/v1/workers") {
      Value arr = Value::array();
      for (const auto& w : *pool.snapshot()) arr.push(w->to_public());
      Value out = Value::object();
      out.set("workers", arr);
      send_simple(cfd, 200, "application/json", dump_json(out), {}, keep);
      return;
    }
    if (req.method == "GET" && p == "/v1/models") {
      Value data = Value::array();
      for (const auto& m : pool.models()) {
        Value e = Value::object();
        e.set("id", Value::string(m));
        e.set("object", Value::string("model"));
        e.set("owned_by", Value::string("infera-b200"));
        data.push(e);
      }
      Value out = Value::object();
      out.set("object", Value::string("list"));
      out.set("data", data);
      send_simple(cfd, 200, "application/json", dump_json(out), {}, keep);
      return;
    }
    if (req.method == "GET" && p == "/metrics") {
      send_simple(cfd, 200, "text/plain; version=0.0.4", metrics_text(), {}, keep);
      return;
    }
    const std::string cv = "/v1/admin/cache-view/";
    if (req.method == "GET" && p.compare(0, cv.size(), cv) == 0) {
      std::string id = p.substr(cv.size());
      int rank = -1;
      auto q = req.query.find("dp_rank=");
      if (q != std::string::npos) rank = std::atoi(req.query.c_str() + q + 8);
      bool known = false;
      for (const auto& w : *pool.snapshot()) known = known || w->worker_id == id;
      if (!known) {
        send_simple(cfd, 404, "application/json", err_json("unknown worker '" + id + "'"), {}, keep);
        return;
      }
      Value hs = Value::array();
      for (uint64_t h : index.view(id, rank, 10000)) hs.push(Value::string(std::to_string(h)));
      Value out = Value::object();
      out.set("worker_id", Value::string(id));
      out.set("dp_rank", rank >= 0 ? Value::integer(rank) : Value());
      out.set("num_blocks", Value::integer(static_cast<int64_t>(index.view_size(id, rank))));
      out.set("block_hashes", hs);
      send_simple(cfd, 200, "application/json", dump_json(out), {}, keep);
      return;
    }
    send_simple(cfd, 404, "application/json", err_json("no route " + req.method + " " + p), {}, keep);
  }

  void conn_loop(int cfd) {
    int one = 1;
    setsockopt(cfd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
    set_timeouts(cfd, 300000, 60000);
    Conn c(cfd);
    while (true) {
      HttpRequest req;
      int r = read_request(c, &req);
      if (r <= 0) {
        if (r < 0) send_simple(cfd, 400, "application/json", err_json("malformed request"), {}, false);
        break;
      }
      handle(cfd, req);
      if (!req.keep_alive) break;
    }
    ::close(cfd);
  }
};

}  // namespace ib

// ---------------------------------------------------------------------------

static void usage() {
  std::fprintf(stderr,
               "ib200_router --port N [--host H] [--discovery-backend etcd|static] [--etcd-endpoint H:P]\n"
               "  [--etcd-prefix P] [--static-workers FILE] [--router-policy kv-aware|round-robin]\n"
               "  [--router-mode auto|direct] [--kv-overlap-weight W] [--kv-prefill-overlap-weight W]\n"
               "  [--kv-decode-overlap-weight W] [--router-tokenizer-path tokenizer.json]\n"
               "  [--request-max-retries N] [--migration-limit N] [--breaker-failure-threshold N]\n"
               "  [--breaker-cooldown-s S] [--breaker-max-cooldown-s S] [--block-size N] [--log-level L]\n");
}

int main(int argc, char** argv) {
  using namespace ib;
  signal(SIGPIPE, SIG_IGN);
  if (argc == 3 && std::strcmp(argv[1], "--print-chain-hashes") == 0) {
    // self-check: token ids on stdin -> chained block hashes on stdout
    std::vector<uint32_t> ids;
    unsigned long long x;
    while (std::scanf("%llu", &x) == 1) ids.push_back(static_cast<uint32_t>(x));
    for (uint64_t h : chain_hashes(ids, std::atoi(argv[2]))) std::printf("%llu\n", static_cast<unsigned long long>(h));
    return 0;
  }
  if (argc == 3 && std::strcmp(argv[1], "--tokenize") == 0) {
    // self-check: one JSON value per stdin line (a string: encode it; an
    // array: chat messages) -> a JSON array of ids, or null if refused
    std::string err;
    auto tk = load_tokenizer_json(argv[2], &err);
    if (!tk) {
      std::fprintf(stderr, "tokenizer: %s\n", err.c_str());
      return 2;
    }
    std::string line;
    char buf[1 << 16];
    while (std::fgets(buf, sizeof buf, stdin)) {
      line += buf;
      if (line.empty() || line.back() != '\n') continue;
      Value v;
      std::vector<uint32_t> ids;
      bool ok = parse_json(line, &v, &err) &&
                (v.is_str() ? tk->try_encode(v.s, &ids) : (v.is_arr() && tk->try_chat(v, &ids)));
      std::string out = ok ? "[" : "null";
      if (ok) {
        for (size_t i = 0; i < ids.size(); ++i) out += (i ? "," : "") + std::to_string(ids[i]);
        out += "]";
      }
      std::printf("%s\n", out.c_str());
      line.clear();
    }
    return 0;
  }
  Config cfg;
  auto env = [](const char* k, const char* d) -> std::string {
    const char* v = std::getenv(k);
    return v && *v ? v : d;
  };
  cfg.discovery = env("INFERA_DISCOVERY_BACKEND", "etcd");
  cfg.etcd_endpoint = env("INFERA_ETCD_ENDPOINT", "");
  cfg.router_mode = env("INFERA_ROUTER_MODE", "auto");
  cfg.tokenizer_path = env("INFERA_ROUTER_TOKENIZER_PATH", "");
  {
    // in-cluster defaults: the API service from the environment, the Pod's
    // service account for token, CA and namespace
    const std::string sa = "/var/run/secrets/kubernetes.io/serviceaccount/";
    auto exists = [](const std::string& f) { return ::access(f.c_str(), R_OK) == 0; };
    const std::string kh = env("KUBERNETES_SERVICE_HOST", "kubernetes.default.svc");
    cfg.k8s.api_url = env("INFERA_K8S_API_URL", ("https://" + kh + ":" + env("KUBERNETES_SERVICE_PORT", "443")).c_str());
    cfg.k8s.selector = env("INFERA_K8S_LABEL_SELECTOR", "");
    cfg.k8s.token_file = exists(sa + "token") ? sa + "token" : "";
    cfg.k8s.ca_file = exists(sa + "ca.crt") ? sa + "ca.crt" : "";
    std::string ns = env("POD_NAMESPACE", "default");
    if (exists(sa + "namespace")) {
      std::ifstream f(sa + "namespace");
      std::string v;
      if (std::getline(f, v) && !v.empty()) ns = v;
    }
    cfg.k8s.namespace_ = ns;
  }
  cfg.max_retries = std::atoi(env("INFERA_REQUEST_MAX_RETRIES", "1").c_str());
  cfg.migration_limit = std::atoi(env("INFERA_MIGRATION_LIMIT", "0").c_str());
  cfg.breaker_threshold = std::atoi(env("INFERA_BREAKER_FAILURE_THRESHOLD", "3").c_str());
  cfg.breaker_cooldown = std::atof(env("INFERA_BREAKER_COOLDOWN_S", "5").c_str());
  cfg.breaker_max_cooldown = std::atof(env("INFERA_BREAKER_MAX_COOLDOWN_S", "60").c_str());
  for (int i = 1; i < argc; ++i) {
    std::string a = argv[i];
    std::string v;
    auto eq = a.find('=');
    if (eq != std::string::npos) {
      v = a.substr(eq + 1);
      a = a.substr(0, eq);
    } else if (i + 1 < argc && std::strncmp(argv[i + 1], "--", 2) != 0) {
      v = argv[++i];
    }
    if (a == "--host") cfg.host = v;
    else if (a == "--port") cfg.port = std::atoi(v.c_str());
    else if (a == "--discovery-backend") cfg.discovery = v;
    else if (a == "--etcd-endpoint") cfg.etcd_endpoint = v;
    else if (a == "--etcd-prefix") cfg.etcd_prefix = v;
    else if (a == "--static-workers") cfg.static_workers = v;
    else if (a == "--router-policy") cfg.policy = v;
    else if (a == "--router-mode") cfg.router_mode = v;
    else if (a == "--router-tokenizer-path") cfg.tokenizer_path = v;
    else if (a == "--kv-overlap-weight") cfg.w = std::atof(v.c_str());
    else if (a == "--kv-prefill-overlap-weight") cfg.wp = std::atof(v.c_str());
    else if (a == "--kv-decode-overlap-weight") cfg.wd = std::atof(v.c_str());
    else if (a == "--request-max-retries") cfg.max_retries = std::atoi(v.c_str());
    else if (a == "--migration-limit") cfg.migration_limit = std::atoi(v.c_str());
    else if (a == "--breaker-failure-threshold") cfg.breaker_threshold = std::atoi(v.c_str());
    else if (a == "--breaker-cooldown-s") cfg.breaker_cooldown = std::atof(v.c_str());
    else if (a == "--breaker-max-cooldown-s") cfg.breaker_max_cooldown = std::atof(v.c_str());
    else if (a == "--block-size") cfg.block_size = std::atoi(v.c_str());
    else if (a == "--log-level") cfg.verbose = v == "debug" || v == "info";
    else if (a == "--help" || a == "-h") { usage(); return 0; }
    else if (a == "--request-transport") cfg.request_transport = v;
    else if (a == "--k8s-label-selector") cfg.k8s.selector = v;
    else if (a == "--k8s-namespace") cfg.k8s.namespace_ = v;
    else if (a == "--k8s-api-url") cfg.k8s.api_url = v;
    else if (a == "--k8s-token-file") cfg.k8s.token_file = v;
    else if (a == "--k8s-ca-file") cfg.k8s.ca_file = v;
    else if (a == "--nats-url") cfg.nats_url = v;
    else if (a == "--nats-idle-timeout") cfg.nats_idle_timeout = std::atof(v.c_str());
    else if (a == "--nats-max-duration") cfg.nats_max_duration = std::atof(v.c_str());
    else if (a == "--router-backend" || a == "--kv-event-transport" ||
             a == "--enable-profiling" || a == "--enable-scaling-api") {
      // accepted for flag compatibility with the Python router; no effect here
    } else {
      std::fprintf(stderr, "[ib200_router] unknown flag %s\n", a.c_str());
      usage();
      return 2;
    }
  }
  if (cfg.policy != "kv-aware" && cfg.policy != "round-robin") {
    std::fprintf(stderr, "[ib200_router] unsupported policy %s\n", cfg.policy.c_str());
    return 2;
  }
  App app(cfg);
  if (cfg.request_transport == "nats") {
    app.nats = std::make_unique<NatsConn>();
    app.nats_idle = cfg.nats_idle_timeout;
    app.nats_max_duration = cfg.nats_max_duration;
    std::string nerr;
    if (!app.nats->connect(cfg.nats_url, &nerr)) {
      std::fprintf(stderr, "[ib200_router] %s\n", nerr.c_str());
      return 2;
    }
  }
  if (cfg.discovery == "etcd") {
    if (cfg.etcd_endpoint.empty()) {
      std::fprintf(stderr, "[ib200_router] --discovery-backend=etcd requires --etcd-endpoint\n");
      return 2;
    }
    app.disc = std::make_unique<EtcdDiscovery>(cfg.etcd_endpoint, cfg.etcd_prefix, &app.pool, &app.gate);
    app.disc->start();
    if (!app.disc->wait_ready(10.0)) std::fprintf(stderr, "[ib200_router] etcd not ready after 10 s; continuing\n");
  } else if (cfg.discovery == "kubernetes" || cfg.discovery == "k8s") {
    if (cfg.k8s.selector.empty()) {
      std::fprintf(stderr, "[ib200_router] --discovery-backend=kubernetes requires --k8s-label-selector\n");
      return 2;
    }
    app.k8s = std::make_unique<K8sDiscovery>(cfg.k8s, &app.pool, &app.gate);
    app.k8s->start();
    if (!app.k8s->wait_ready(10.0))
      std::fprintf(stderr, "[ib200_router] kubernetes API not ready after 10 s; continuing\n");
  } else if (cfg.discovery == "static") {
    std::string err;
    if (!cfg.static_workers.empty() && !load_static_workers(cfg.static_workers, &app.pool, &err)) {
      std::fprintf(stderr, "[ib200_router] %s\n", err.c_str());
      return 2;
    }
  } else {
    std::fprintf(stderr, "[ib200_router] discovery backend %s is served by the Python router\n",
                 cfg.discovery.c_str());
    return 2;
  }
  int lfd = tcp_listen(cfg.host, cfg.port);
  if (lfd < 0) {
    std::fprintf(stderr, "[ib200_router] cannot listen on %s:%d\n", cfg.host.c_str(), cfg.port);
    return 1;
  }
  std::fprintf(stderr, "[ib200_router] listening on %s:%d (policy %s, mode %s)\n", cfg.host.c_str(), cfg.port,
               cfg.policy.c_str(), cfg.router_mode.c_str());
  while (true) {
    int cfd = ::accept4(lfd, nullptr, nullptr, SOCK_CLOEXEC);
    if (cfd < 0) {
      if (errno == EINTR || errno == ECONNABORTED || errno == EMFILE) continue;
      break;
    }
    std::thread(&App::conn_loop, &app, cfd).detach();
  }
  return 0;
}
