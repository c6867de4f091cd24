// HTTP/1.1 server core for the coordinator (reference coordinator/src/main.rs:126-137 serves the same
// API with axum): POSIX sockets, one poller thread (accepts, and watches idle keep-alive connections),
// a fixed worker pool that serves a connection only while it has a request, Content-Length bodies up to a configurable cap (512 MB in the reference), permissive
// CORS (CorsLayer::permissive) including OPTIONS preflight. Requests are handed to a C callback that
// routes them and fills the response through dtr_http_respond().
#include <arpa/inet.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <sys/socket.h>
#include <unistd.h>

#include <fcntl.h>

#include <algorithm>
#include <chrono>
#include <atomic>
#include <cerrno>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#define DT_API extern "C" __attribute__((visibility("default")))

namespace {

struct Response {
  int status = 200;
  std::string content_type = "application/json";
  std::string body;
};

using Handler = void (*)(void* ctx, const char* method, const char* path, const char* body, long long body_len,
                         void* response);

struct Conn {
  int fd = -1;
  std::string buf;  // bytes read past the last served request
  std::chrono::steady_clock::time_point idle_since;
};

struct Server {
  int fd = -1;
  int port = 0;
  Handler handler = nullptr;
  void* ctx = nullptr;
  long long max_body = 512LL << 20;
  std::atomic<bool> stop{false};
  std::thread acceptor;
  std::vector<std::thread> workers;
  std::mutex mu;
  std::condition_variable cv;
  std::deque<Conn*> queue;      // connections with data, waiting for a worker
  std::vector<Conn*> idle;      // keep-alive connections watched by the poller
  int wake[2] = {-1, -1};       // self-pipe: a worker parked a connection
  std::atomic<long long> served{0};
};

const char* reason(int s) {
  switch (s) {
    case 200: return "OK";
    case 201: return "Created";
    case 204: return "No Content";
    case 400: return "Bad Request";
    case 401: return "Unauthorized";
    case 404: return "Not Found";
    case 405: return "Method Not Allowed";
    case 411: return "Length Required";
    case 413: return "Payload Too Large";
    case 500: return "Internal Server Error";
    case 503: return "Service Unavailable";
    default: return "Status";
  }
}

bool send_all(int fd, const char* p, size_t n) {
  while (n) {
    ssize_t w = ::send(fd, p, n, MSG_NOSIGNAL);
    if (w < 0) {
      if (errno == EINTR) continue;
      return false;
    }
    p += w;
    n -= (size_t)w;
  }
  return true;
}

// Read until "\r\n\r\n" (headers) with a poll timeout; leftover bytes stay in `buf`.
bool read_headers(int fd, std::string& buf, size_t& hdr_end, std::atomic<bool>& stop) {
  int idle = 0;
  while (true) {
    size_t p = buf.find("\r\n\r\n");
    if (p != std::string::npos) {
      hdr_end = p + 4;
      return true;
    }
    if (buf.size() > (1 << 20)) return false;
    struct pollfd pf{fd, POLLIN, 0};
    int r = poll(&pf, 1, 200);
    if (stop.load()) return false;
    if (r == 0) {
      if (++idle > 300) return false;  // 60 s idle keep-alive limit
      continue;
    }
    if (r < 0) {
      if (errno == EINTR) continue;
      return false;
    }
    char tmp[65536];
    ssize_t n = ::recv(fd, tmp, sizeof tmp, 0);
    if (n <= 0) return false;
    buf.append(tmp, (size_t)n);
  }
}

std::string lower(std::string s) {
  std::transform(s.begin(), s.end(), s.begin(), [](unsigned char c) { return (char)std::tolower(c); });
  return s;
}

void respond(int fd, const Response& r, bool keep_alive) {
  std::string h = "HTTP/1.1 " + std::to_string(r.status) + " " + reason(r.status) + "\r\n";
  h += "Content-Type: " + r.content_type + "\r\n";
  h += "Content-Length: " + std::to_string(r.body.size()) + "\r\n";
  h += "Access-Control-Allow-Origin: *\r\n";
  h += "Access-Control-Allow-Methods: *\r\nAccess-Control-Allow-Headers: *\r\n";
  h += keep_alive ? "Connection: keep-alive\r\n\r\n" : "Connection: close\r\n\r\n";
  if (send_all(fd, h.data(), h.size())) send_all(fd, r.body.data(), r.body.size());
}

// Serve the requests available on one connection. Returns true if the connection stays open
// (keep-alive) and should go back to the poller, false if it was closed.
bool serve_connection(Server* s, Conn* cn) {
  const int fd = cn->fd;
  std::string& buf = cn->buf;
  do {
    size_t hend = 0;
    if (!read_headers(fd, buf, hend, s->stop)) return false;
    std::string head = buf.substr(0, hend);
    buf.erase(0, hend);
    size_t le = head.find("\r\n");
    std::string line = head.substr(0, le);
    size_t sp1 = line.find(' '), sp2 = line.rfind(' ');
    if (sp1 == std::string::npos || sp2 == sp1) {
      respond(fd, Response{400, "text/plain", "bad request line"}, false);
      return false;
    }
    std::string method = line.substr(0, sp1), path = line.substr(sp1 + 1, sp2 - sp1 - 1);
    std::string version = line.substr(sp2 + 1);
    long long clen = 0;
    bool keep_alive = version == "HTTP/1.1", chunked = false;
    size_t pos = le + 2;
    while (pos < head.size()) {
      size_t e = head.find("\r\n", pos);
      if (e == std::string::npos || e == pos) break;
      std::string hl = head.substr(pos, e - pos);
      pos = e + 2;
      size_t c = hl.find(':');
      if (c == std::string::npos) continue;
      std::string k = lower(hl.substr(0, c)), v = hl.substr(c + 1);
      v.erase(0, v.find_first_not_of(" \t"));
      if (k == "content-length") clen = atoll(v.c_str());
      else if (k == "connection") keep_alive = lower(v).find("close") == std::string::npos &&
                                               (version == "HTTP/1.1" || lower(v).find("keep-alive") != std::string::npos);
      else if (k == "transfer-encoding" && lower(v).find("chunked") != std::string::npos) chunked = true;
    }
    if (chunked) {
      respond(fd, Response{411, "text/plain", "chunked bodies are not supported; send Content-Length"}, false);
      return false;
    }
    if (clen > s->max_body) {
      respond(fd, Response{413, "text/plain", "body exceeds limit"}, false);
      return false;
    }
    while ((long long)buf.size() < clen) {
      struct pollfd pf{fd, POLLIN, 0};
      int r = poll(&pf, 1, 30000);
      if (r <= 0) return false;
      char tmp[1 << 16];
      ssize_t n = ::recv(fd, tmp, sizeof tmp, 0);
      if (n <= 0) return false;
      buf.append(tmp, (size_t)n);
    }
    std::string body = buf.substr(0, (size_t)clen);
    buf.erase(0, (size_t)clen);
    Response r;
    if (method == "OPTIONS") {
      r.status = 204;
      r.content_type = "text/plain";
    } else {
      s->handler(s->ctx, method.c_str(), path.c_str(), body.data(), (long long)body.size(), &r);
    }
    respond(fd, r, keep_alive);
    s->served++;
    if (!keep_alive) return false;
  } while (buf.find("\r\n\r\n") != std::string::npos);  // pipelined request already buffered
  return true;
}

void close_conn(Conn* c) {
  ::close(c->fd);
  delete c;
}

void park(Server* s, Conn* c) {
  {
    std::lock_guard<std::mutex> lk(s->mu);
    c->idle_since = std::chrono::steady_clock::now();
    s->idle.push_back(c);
  }
  char b = 1;
  (void)!::write(s->wake[1], &b, 1);
}

void worker_loop(Server* s) {
  while (true) {
    Conn* c;
    {
      std::unique_lock<std::mutex> lk(s->mu);
      s->cv.wait(lk, [&] { return s->stop.load() || !s->queue.empty(); });
      if (s->stop.load() && s->queue.empty()) return;
      c = s->queue.front();
      s->queue.pop_front();
    }
    if (serve_connection(s, c) && !s->stop.load()) park(s, c);
    else close_conn(c);
  }
}

// Poller: accepts connections and watches idle keep-alive connections; a connection with data (or a
// hang-up) is handed to a worker, so idle clients never hold a worker thread.
void accept_loop(Server* s) {
  std::vector<pollfd> pfs;
  std::vector<Conn*> watched;
  while (!s->stop.load()) {
    pfs.clear();
    watched.clear();
    pfs.push_back({s->fd, POLLIN, 0});
    pfs.push_back({s->wake[0], POLLIN, 0});
    {
      std::lock_guard<std::mutex> lk(s->mu);
      auto now = std::chrono::steady_clock::now();
      std::vector<Conn*> keep;
      for (Conn* c : s->idle) {
        if (now - c->idle_since > std::chrono::seconds(60)) { close_conn(c); continue; }
        keep.push_back(c);
      }
      s->idle.swap(keep);
      for (Conn* c : s->idle) {
        pfs.push_back({c->fd, POLLIN, 0});
        watched.push_back(c);
      }
    }
    int r = poll(pfs.data(), pfs.size(), 100);
    if (r <= 0) continue;
    if (pfs[1].revents) {
      char tmp[256];
      while (::read(s->wake[0], tmp, sizeof tmp) > 0) {}
    }
    std::vector<Conn*> ready;
    if (pfs[0].revents & POLLIN) {
      int c = ::accept(s->fd, nullptr, nullptr);
      if (c >= 0) {
        int one = 1;
        setsockopt(c, IPPROTO_TCP, TCP_NODELAY, &one, sizeof one);
        Conn* cn = new Conn;
        cn->fd = c;
        std::lock_guard<std::mutex> lk(s->mu);
        cn->idle_since = std::chrono::steady_clock::now();
        s->idle.push_back(cn);  // served once it has data
      }
    }
    for (size_t i = 2; i < pfs.size(); ++i)
      if (pfs[i].revents) ready.push_back(watched[i - 2]);
    if (!ready.empty()) {
      std::lock_guard<std::mutex> lk(s->mu);
      std::vector<Conn*> keep;
      for (Conn* c : s->idle)
        if (std::find(ready.begin(), ready.end(), c) == ready.end()) keep.push_back(c);
      s->idle.swap(keep);
      for (Conn* c : ready) s->queue.push_back(c);
    }
    for (size_t i = 0; i < ready.size(); ++i) s->cv.notify_one();
  }
}

}  // namespace

// Start serving on host:port (port 0 = ephemeral; read back with dtr_http_port). Returns a handle or null.
DT_API void* dtr_http_start(const char* host, int port, int nthreads, long long max_body, Handler h, void* ctx) {
  auto* s = new Server;
  s->handler = h;
  s->ctx = ctx;
  if (max_body > 0) s->max_body = max_body;
  if (pipe(s->wake) != 0) { delete s; return nullptr; }
  fcntl(s->wake[0], F_SETFL, O_NONBLOCK);
  fcntl(s->wake[1], F_SETFL, O_NONBLOCK);
  s->fd = ::socket(AF_INET, SOCK_STREAM, 0);
  int one = 1;
  setsockopt(s->fd, SOL_SOCKET, SO_REUSEADDR, &one, sizeof one);
  sockaddr_in a{};
  a.sin_family = AF_INET;
  a.sin_port = htons((uint16_t)port);
  if (!host || !*host || strcmp(host, "0.0.0.0") == 0) a.sin_addr.s_addr = INADDR_ANY;
  else inet_pton(AF_INET, host, &a.sin_addr);
  if (::bind(s->fd, (sockaddr*)&a, sizeof a) != 0 || ::listen(s->fd, 256) != 0) {
    ::close(s->fd);
    ::close(s->wake[0]);
    ::close(s->wake[1]);
    delete s;
    return nullptr;
  }
  socklen_t al = sizeof a;
  getsockname(s->fd, (sockaddr*)&a, &al);
  s->port = ntohs(a.sin_port);
  if (nthreads < 1) nthreads = 8;
  for (int i = 0; i < nthreads; ++i) s->workers.emplace_back(worker_loop, s);
  s->acceptor = std::thread(accept_loop, s);
  return s;
}

DT_API int dtr_http_port(void* h) { return static_cast<Server*>(h)->port; }
DT_API long long dtr_http_served(void* h) { return static_cast<Server*>(h)->served.load(); }

DT_API void dtr_http_respond(void* resp, int status, const char* content_type, const void* body, long long n) {
  auto* r = static_cast<Response*>(resp);
  r->status = status;
  if (content_type) r->content_type = content_type;
  r->body.assign((const char*)body, (size_t)n);
}

DT_API void dtr_http_stop(void* h) {
  auto* s = static_cast<Server*>(h);
  if (!s) return;
  s->stop = true;
  s->cv.notify_all();
  if (s->acceptor.joinable()) s->acceptor.join();
  for (auto& t : s->workers)
    if (t.joinable()) t.join();
  {
    std::lock_guard<std::mutex> lk(s->mu);
    for (Conn* c : s->queue) close_conn(c);
    for (Conn* c : s->idle) close_conn(c);
    s->queue.clear();
    s->idle.clear();
  }
  ::close(s->fd);
  ::close(s->wake[0]);
  ::close(s->wake[1]);
  delete s;
}
