// Fleet discovery (see discovery.h). The etcd flow follows the Python
// registry (infera_b200/common/discovery.py), itself the flow of the
// reference's infera/common/registry.py and rust/router/src/discovery.rs:24.
#include "discovery.h"

#include <poll.h>
#include <unistd.h>

#include <cctype>
#include <chrono>
#include <cstdio>
#include <iterator>
#include <fstream>
#include <set>
#include <sstream>

#include "net.h"

namespace ib {

static void logf(const char* fmt, const std::string& a) {
  std::fprintf(stderr, "[ib200_router] ");
  std::fprintf(stderr, fmt, a.c_str());
  std::fprintf(stderr, "\n");
}

bool CanaryGate::admit(const Worker& w, std::string* why) {
  const Value* kv = w.record.get("kv");
  const Value* c = kv ? kv->get("tokenizer_canary") : nullptr;
  if (!c) return true;
  std::string cj = dump_json(*c);
  std::lock_guard<std::mutex> g(mu_);
  auto it = ref_.find(w.model_name);
  if (it == ref_.end() || it->second.second == w.worker_id) {
    ref_[w.model_name] = {cj, w.worker_id};
    return true;
  }
  if (it->second.first != cj) {
    *why = "tokenizer canary of " + w.worker_id + " differs from first-registered " + it->second.second;
    return false;
  }
  return true;
}

void CanaryGate::forget_if_absent(const Pool& pool) {
  auto snap = pool.snapshot();
  std::lock_guard<std::mutex> g(mu_);
  for (auto it = ref_.begin(); it != ref_.end();) {
    bool any = false;
    for (const auto& w : *snap) any = any || w->model_name == it->first;
    it = any ? std::next(it) : ref_.erase(it);
  }
}

static std::string prefix_end(const std::string& p) {
  std::string e = p;
  for (int i = static_cast<int>(e.size()) - 1; i >= 0; --i) {
    unsigned char c = static_cast<unsigned char>(e[i]);
    if (c < 0xFF) {
      e[i] = static_cast<char>(c + 1);
      e.resize(i + 1);
      return e;
    }
  }
  return std::string(1, '\0');
}

void EtcdDiscovery::start() { th_ = std::thread(&EtcdDiscovery::run, this); }

void EtcdDiscovery::stop() {
  stop_ = true;
  if (th_.joinable()) th_.join();
}

bool EtcdDiscovery::wait_ready(double timeout_s) {
  auto t0 = std::chrono::steady_clock::now();
  while (!ready_) {
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > timeout_s) return false;
    std::this_thread::sleep_for(std::chrono::milliseconds(20));
  }
  return true;
}

std::string EtcdDiscovery::post(const std::string& path, const std::string& body, int* status) {
  Url u;
  std::string ep = endpoint_.find("://") == std::string::npos ? "http://" + endpoint_ : endpoint_;
  *status = 0;
  if (!parse_url(ep, &u)) return "";
  int fd = tcp_connect(u.host, u.port, 3000);
  if (fd < 0) return "";
  set_timeouts(fd, 10000, 10000);
  std::string req = "POST " + path + " HTTP/1.1\r\nHost: " + u.host + "\r\nContent-Type: application/json\r\n"
                    "Content-Length: " + std::to_string(body.size()) + "\r\nConnection: close\r\n\r\n" + body;
  std::string out;
  if (write_all(fd, req)) {
    Conn c(fd);
    HttpResponseHead h;
    if (read_response_head(c, &h)) {
      *status = h.status;
      BodyReader br(c, h);
      while (br.next(&out)) {
      }
    }
  }
  ::close(fd);
  return out;
}

void EtcdDiscovery::apply_put(const std::string& value_b64) {
  Value rec;
  std::string err;
  if (!parse_json(base64_decode(value_b64), &rec, &err)) {
    logf("skipping malformed worker record: %s", err);
    return;
  }
  Worker w;
  if (!Worker::from_json(rec, &w, &err)) {
    logf("skipping worker record: %s", err);
    return;
  }
  std::string why;
  if (!gate_->admit(w, &why)) {
    rejected++;
    logf("refused: %s", why);
    return;
  }
  pool_->upsert(w);
}

bool EtcdDiscovery::snapshot() {
  Value body = Value::object();
  body.set("key", Value::string(base64_encode(prefix_)));
  body.set("range_end", Value::string(base64_encode(prefix_end(prefix_))));
  int st = 0;
  std::string resp = post("/v3/kv/range", dump_json(body), &st);
  if (st != 200) return false;
  Value v;
  std::string err;
  if (!parse_json(resp, &v, &err)) return false;
  if (const Value* h = v.get("header"))
    if (const Value* r = h->get("revision")) rev_ = r->is_str() ? std::atoll(r->s.c_str()) : r->as_int();
  std::set<std::string> seen;
  if (const Value* kvs = v.get("kvs"))
    for (const auto& kv : kvs->arr()) {
      const Value* val = kv.get("value");
      if (!val || !val->is_str()) continue;
      Value rec;
      if (parse_json(base64_decode(val->s), &rec, &err)) {
        const Value* id = rec.get("worker_id");
        if (id && id->is_str()) seen.insert(id->s);
      }
      apply_put(val->s);
    }
  auto snap = pool_->snapshot();
  for (const auto& w : *snap)
    if (!seen.count(w->worker_id)) pool_->remove(w->worker_id);
  gate_->forget_if_absent(*pool_);
  snapshots++;
  ready_ = true;
  return true;
}

void EtcdDiscovery::watch() {
  Url u;
  std::string ep = endpoint_.find("://") == std::string::npos ? "http://" + endpoint_ : endpoint_;
  if (!parse_url(ep, &u)) return;
  int fd = tcp_connect(u.host, u.port, 3000);
  if (fd < 0) return;
  Value cr = Value::object();
  cr.set("key", Value::string(base64_encode(prefix_)));
  cr.set("range_end", Value::string(base64_encode(prefix_end(prefix_))));
  cr.set("start_revision", Value::string(std::to_string(rev_ + 1)));
  Value body = Value::object();
  body.set("create_request", cr);
  std::string b = dump_json(body);
  std::string req = "POST /v3/watch HTTP/1.1\r\nHost: " + u.host + "\r\nContent-Type: application/json\r\n"
                    "Content-Length: " + std::to_string(b.size()) + "\r\n\r\n" + b;
  if (!write_all(fd, req)) { ::close(fd); return; }
  Conn c(fd);
  HttpResponseHead h;
  set_timeouts(fd, 10000, 10000);
  if (!read_response_head(c, &h) || h.status != 200) { ::close(fd); return; }
  BodyReader br(c, h);
  std::string buf;
  while (!stop_) {
    if (c.buffered() == 0) {
      pollfd pf{fd, POLLIN, 0};
      int r = ::poll(&pf, 1, 250);
      if (r == 0) continue;
      if (r < 0) break;
    }
    if (!br.next(&buf)) break;
    size_t nl;
    while ((nl = buf.find('\n')) != std::string::npos) {
      std::string line = buf.substr(0, nl);
      buf.erase(0, nl + 1);
      if (line.find_first_not_of(" \r\t") == std::string::npos) continue;
      Value msg;
      std::string err;
      if (!parse_json(line, &msg, &err)) continue;
      const Value* result = msg.get("result");
      if (!result) result = &msg;
      const Value* evs = result->get("events");
      if (!evs) continue;
      for (const auto& ev : evs->arr()) {
        const Value* kv = ev.get("kv");
        if (!kv) continue;
        events++;
        const Value* type = ev.get("type");
        const Value* key = kv->get("key");
        if (type && type->is_str() && type->s == "DELETE") {
          std::string k = key && key->is_str() ? base64_decode(key->s) : "";
          std::string id = k.compare(0, prefix_.size(), prefix_) == 0 ? k.substr(prefix_.size()) : k;
          pool_->remove(id);
          gate_->forget_if_absent(*pool_);
        } else if (const Value* val = kv->get("value"); val && val->is_str()) {
          apply_put(val->s);
        }
        if (const Value* mr = kv->get("mod_revision")) {
          int64_t r = mr->is_str() ? std::atoll(mr->s.c_str()) : mr->as_int();
          if (r > rev_) rev_ = r;
        }
      }
    }
  }
  ::close(fd);
}

void EtcdDiscovery::run() {
  while (!stop_) {
    if (snapshot()) watch();
    for (int i = 0; i < 10 && !stop_; ++i) std::this_thread::sleep_for(std::chrono::milliseconds(100));
  }
}

// ---------------------------------------------------------------------------
// Kubernetes (flow of infera_b200/common/discovery_k8s.py, itself the role of
// the reference's rust/router/src/discovery_k8s.rs:59)

static const char* const kWorkerInfoAnnotation = "infera.amd.com/worker-info";

struct K8sDiscovery::Stream {
  int fd = -1;
  TlsSession* tls = nullptr;
  Conn conn;
  HttpResponseHead head;
  ~Stream() {
    tls_free(tls);
    if (fd >= 0) ::close(fd);
  }
};

static std::string url_escape(const std::string& s) {
  static const char* hex = "0123456789ABCDEF";
  std::string out;
  for (unsigned char c : s) {
    if (std::isalnum(c) || c == '-' || c == '_' || c == '.' || c == '~') {
      out.push_back(static_cast<char>(c));
    } else {
      out.push_back('%');
      out.push_back(hex[c >> 4]);
      out.push_back(hex[c & 15]);
    }
  }
  return out;
}

bool K8sDiscovery::open_get(const std::string& path_query, Stream* st, int* status) {
  *status = 0;
  std::string rest = cfg_.api_url;
  bool tls = false;
  if (rest.compare(0, 8, "https://") == 0) {
    tls = true;
    rest = rest.substr(8);
  } else if (rest.compare(0, 7, "http://") == 0) {
    rest = rest.substr(7);
  }
  const size_t slash = rest.find('/');
  std::string hostport = slash == std::string::npos ? rest : rest.substr(0, slash);
  std::string base_path = slash == std::string::npos ? "" : rest.substr(slash);
  while (!base_path.empty() && base_path.back() == '/') base_path.pop_back();
  std::string host = hostport;
  int port = tls ? 443 : 80;
  const size_t colon = hostport.rfind(':');
  if (colon != std::string::npos && hostport.find(']') == std::string::npos) {
    host = hostport.substr(0, colon);
    port = std::atoi(hostport.c_str() + colon + 1);
  }
  st->fd = tcp_connect(host, port, 3000);
  if (st->fd < 0) return false;
  set_timeouts(st->fd, 10000, 10000);
  std::string err;
  if (tls) {
    st->tls = tls_connect(st->fd, host, cfg_.ca_file, &err);
    if (st->tls == nullptr) {
      logf("kubernetes: %s", err);
      return false;
    }
  }
  std::string auth;
  if (!cfg_.token_file.empty()) {
    std::ifstream f(cfg_.token_file);
    std::string tok((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    while (!tok.empty() && (tok.back() == '\n' || tok.back() == '\r' || tok.back() == ' ')) tok.pop_back();
    if (!tok.empty()) auth = "Authorization: Bearer " + tok + "\r\n";
  }
  const std::string req = "GET " + base_path + path_query + " HTTP/1.1\r\nHost: " + hostport +
                          "\r\nAccept: application/json\r\n" + auth + "Connection: close\r\n\r\n";
  if (!(tls ? tls_write_all(st->tls, req) : write_all(st->fd, req))) return false;
  st->conn.reset(st->fd);
  st->conn.set_tls(st->tls);
  if (!read_response_head(st->conn, &st->head)) return false;
  *status = st->head.status;
  return true;
}

void K8sDiscovery::handle(const std::string& kind, const Value& pod) {
  const Value* meta = pod.get("metadata");
  const Value* name_v = meta ? meta->get("name") : nullptr;
  if (!name_v || !name_v->is_str()) return;
  const std::string name = name_v->s;
  const Value* ann = meta->get("annotations");
  const Value* raw = ann ? ann->get(kWorkerInfoAnnotation) : nullptr;
  Value rec;
  std::string err;
  const bool has_rec = raw && raw->is_str() && parse_json(raw->s, &rec, &err);
  auto drop = [&]() {
    auto it = pod_worker_.find(name);
    if (it != pod_worker_.end()) {
      pool_->remove(it->second);
      pod_worker_.erase(it);
      gate_->forget_if_absent(*pool_);
    }
  };
  if (kind == "DELETED" || !has_rec) {
    if (raw && !has_rec) logf("pod %s has a malformed worker record", name);
    drop();
    return;
  }
  Worker w;
  if (!Worker::from_json(rec, &w, &err)) {
    logf("pod %s: bad worker record", name);
    return;
  }
  auto old = pod_worker_.find(name);
  if (old != pod_worker_.end() && old->second != w.worker_id) drop();
  std::string why;
  if (!gate_->admit(w, &why)) {
    rejected++;
    logf("refused: %s", why);
    return;
  }
  const Value* del = meta->get("deletionTimestamp");
  // terminating: kept (in-flight streams finish) but no longer routed
  w.status = del && !del->is_null() ? "draining" : "active";
  pool_->upsert(w);
  pod_worker_[name] = w.worker_id;
}

bool K8sDiscovery::relist() {
  Stream st;
  int status = 0;
  const std::string path = "/api/v1/namespaces/" + url_escape(cfg_.namespace_) +
                           "/pods?labelSelector=" + url_escape(cfg_.selector);
  if (!open_get(path, &st, &status) || status != 200) {
    if (status) logf("kubernetes list: HTTP %s", std::to_string(status));
    return false;
  }
  std::string body;
  BodyReader br(st.conn, st.head);
  while (br.next(&body)) {
  }
  if (br.error()) return false;
  Value v;
  std::string err;
  if (!parse_json(body, &v, &err)) return false;
  if (const Value* m = v.get("metadata"))
    if (const Value* rv = m->get("resourceVersion"); rv && rv->is_str()) rv_ = rv->s;
  std::set<std::string> seen;
  if (const Value* items = v.get("items"))
    for (const auto& pod : items->arr()) {
      const Value* meta = pod.get("metadata");
      const Value* nm = meta ? meta->get("name") : nullptr;
      if (nm && nm->is_str()) seen.insert(nm->s);
      handle("ADDED", pod);
    }
  std::vector<std::string> gone;
  for (const auto& kv : pod_worker_)
    if (!seen.count(kv.first)) gone.push_back(kv.first);
  for (const auto& name : gone) {
    pool_->remove(pod_worker_[name]);
    pod_worker_.erase(name);
  }
  gate_->forget_if_absent(*pool_);
  relists++;
  ready_ = true;
  return true;
}

void K8sDiscovery::watch() {
  Stream st;
  int status = 0;
  const std::string path = "/api/v1/namespaces/" + url_escape(cfg_.namespace_) + "/pods?labelSelector=" +
                           url_escape(cfg_.selector) + "&watch=true&allowWatchBookmarks=true&resourceVersion=" +
                           url_escape(rv_);
  if (!open_get(path, &st, &status) || status != 200) return;
  BodyReader br(st.conn, st.head);
  std::string buf;
  while (!stop_) {
    if (st.conn.buffered() == 0 && (st.tls == nullptr || tls_pending(st.tls) == 0)) {
      pollfd pf{st.fd, POLLIN, 0};
      const int r = ::poll(&pf, 1, 250);
      if (r == 0) continue;
      if (r < 0) break;
    }
    if (!br.next(&buf)) break;
    size_t nl;
    while ((nl = buf.find('\n')) != std::string::npos) {
      std::string line = buf.substr(0, nl);
      buf.erase(0, nl + 1);
      if (line.find_first_not_of(" \r\t") == std::string::npos) continue;
      Value ev;
      std::string err;
      if (!parse_json(line, &ev, &err)) continue;
      const Value* type = ev.get("type");
      const Value* obj = ev.get("object");
      const std::string kind = type && type->is_str() ? type->s : "MODIFIED";
      if (kind == "ERROR") return;  // e.g. 410 Gone: re-list
      if (obj)
        if (const Value* m = obj->get("metadata"))
          if (const Value* rv = m->get("resourceVersion"); rv && rv->is_str()) rv_ = rv->s;
      if (kind == "BOOKMARK" || !obj) continue;
      events++;
      handle(kind, *obj);
    }
  }
}

void K8sDiscovery::start() { th_ = std::thread(&K8sDiscovery::run, this); }

void K8sDiscovery::stop() {
  stop_ = true;
  if (th_.joinable()) th_.join();
}

bool K8sDiscovery::wait_ready(double timeout_s) {
  auto t0 = std::chrono::steady_clock::now();
  while (!ready_) {
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > timeout_s) return false;
    std::this_thread::sleep_for(std::chrono::milliseconds(20));
  }
  return true;
}

void K8sDiscovery::run() {
  while (!stop_) {
    if (relist()) watch();
    for (int i = 0; i < 10 && !stop_; ++i) std::this_thread::sleep_for(std::chrono::milliseconds(100));
  }
}

bool load_static_workers(const std::string& path, Pool* pool, std::string* err) {
  std::ifstream f(path);
  if (!f) {
    *err = "cannot open " + path;
    return false;
  }
  std::stringstream ss;
  ss << f.rdbuf();
  Value v;
  if (!parse_json(ss.str(), &v, err)) return false;
  const Value* list = v.is_arr() ? &v : v.get("workers");
  if (!list) {
    *err = "expected a list of worker records";
    return false;
  }
  for (const auto& rec : list->arr()) {
    Worker w;
    if (!Worker::from_json(rec, &w, err)) return false;
    pool->upsert(w);
  }
  return true;
}

}  // namespace ib
