// HTTP/1.1 server core for the coordinator (reference coordinator/src/main.rs:126-137 serves the same
// API with axum): POSIX sockets, one acceptor thread, a fixed worker pool, persistent (keep-alive)
// connections, Content-Length bodies up to a configurable cap (512 MB in the reference), permissive
// CORS (CorsLayer::permissive) including OPTIONS preflight. Requests are handed to a C callback that
// routes them and fills the response through dtr_http_respond().
#include <arpa/inet.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <sys/socket.h>
#include <unistd.h>

#include <algorithm>
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
  std::deque<int> queue;
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

void serve_connection(Server* s, int fd) {
  std::string buf;
  while (!s->stop.load()) {
    size_t hend = 0;
    if (!read_headers(fd, buf, hend, s->stop)) break;
    std::string head = buf.substr(0, hend);
    buf.erase(0, hend);
    size_t le = head.find("\r\n");
    std::string line = head.substr(0, le);
    size_t sp1 = line.find(' '), sp2 = line.rfind(' ');
    if (sp1 == std::string::npos || sp2 == sp1) {
      respond(fd, Response{400, "text/plain", "bad request line"}, false);
      break;
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
      break;
    }
    if (clen > s->max_body) {
      respond(fd, Response{413, "text/plain", "body exceeds limit"}, false);
      break;
    }
    while ((long long)buf.size() < clen) {
      char tmp[1 << 16];
      ssize_t n = ::recv(fd, tmp, sizeof tmp, 0);
      if (n <= 0) { keep_alive = false; break; }
      buf.append(tmp, (size_t)n);
    }
    if ((long long)buf.size() < clen) break;
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
    if (!keep_alive) break;
  }
  ::close(fd);
}

void worker_loop(Server* s) {
  while (true) {
    int fd;
    {
      std::unique_lock<std::mutex> lk(s->mu);
      s->cv.wait(lk, [&] { return s->stop.load() || !s->queue.empty(); });
      if (s->stop.load() && s->queue.empty()) return;
      fd = s->queue.front();
      s->queue.pop_front();
    }
    serve_connection(s, fd);
  }
}

void accept_loop(Server* s) {
  while (!s->stop.load()) {
    struct pollfd pf{s->fd, POLLIN, 0};
    int r = poll(&pf, 1, 100);
    if (r <= 0) continue;
    int c = ::accept(s->fd, nullptr, nullptr);
    if (c < 0) continue;
    int one = 1;
    setsockopt(c, IPPROTO_TCP, TCP_NODELAY, &one, sizeof one);
    {
      std::lock_guard<std::mutex> lk(s->mu);
      s->queue.push_back(c);
    }
    s->cv.notify_one();
  }
}

}  // namespace

// Start serving on host:port (port 0 = ephemeral; read back with dtr_http_port). Returns a handle or null.
DT_API void* dtr_http_start(const char* host, int port, int nthreads, long long max_body, Handler h, void* ctx) {
  auto* s = new Server;
  s->handler = h;
  s->ctx = ctx;
  if (max_body > 0) s->max_body = max_body;
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
    for (int fd : s->queue) ::close(fd);
    s->queue.clear();
  }
  ::close(s->fd);
  delete s;
}
