// Self-test of the C++ runtime through its C API, built together with the runtime sources under
// AddressSanitizer + UndefinedBehaviorSanitizer and, separately, ThreadSanitizer
// (distrain_b200/_build.py build_runtime_selftest; run by tests/test_runtime_sanitizers.py).
//
//   http     a server with 4 workers and 8 client threads issuing keep-alive requests with bodies of
//            varying size (the accept / idle / queue hand-off between threads is what TSan watches),
//            plus a malformed request and a body above the limit
//   codecs   safetensors save -> open -> read back, DTZ1 encode -> decode (int8 and fp32), SipHash /
//            splitmix64 / shard assignment determinism, zstd round trip when the library is present
//   sched    push acceptance / merge trigger / round-time rules of the coordinator
//   loader   three uint16 shard files: synchronous reads across shard boundaries with wrap-around, then
//            the prefetch thread filling caller buffers while this thread consumes them
//
// Exit code 0 = all checks passed; a failed check prints its line and exits 1; the sanitizers abort on
// their own findings.
#include <arpa/inet.h>
#include <netinet/in.h>
#include <sys/socket.h>
#include <unistd.h>

#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

extern "C" {
using Handler = void (*)(void*, const char*, const char*, const char*, long long, void*);
void* dtr_http_start(const char*, int, int, long long, Handler, void*);
int dtr_http_port(void*);
long long dtr_http_served(void*);
void dtr_http_respond(void*, int, const char*, const void*, long long);
void dtr_http_stop(void*);
int dtr_st_save(const char*, int, const char* const*, const int*, const long long*, const float* const*, const char*,
                void**);
void* dtr_st_open_bytes(const void*, long long);
void dtr_st_close(void*);
int dtr_st_count(void*);
const char* dtr_st_name(void*, int);
long long dtr_st_read_f32(void*, int, float*, long long);
long long dtr_blob_size(void*);
const void* dtr_blob_data(void*);
void dtr_blob_free(void*);
void* dtr_dtz_encode(long long, long long, const int*, const signed char*, const float*, const float*, int, int);
void* dtr_dtz_decode_dense(const void*, long long);
int dtr_zstd_available();
void* dtr_zstd_compress(const void*, long long, int);
void* dtr_zstd_decompress(const void*, long long);
unsigned long long dtr_siphash13(const void*, long long);
unsigned long long dtr_splitmix64(unsigned long long);
long long dtr_shard_assignment(const char*, unsigned long long, long long, long long, long long*);
void* dtr_loader_open(const char*, long long, long long, int);
int dtr_loader_next(void*, int32_t*, long long);
void dtr_loader_reset(void*);
int dtr_loader_start_prefetch(void*, int32_t**, int);
int dtr_loader_acquire(void*, int);
void dtr_loader_release(void*, int);
void dtr_loader_close(void*);
int dts_accept_push(long long, long long, int, int, const char* const*, const long long*, const char*, long long,
                    double, double, double*, char*, int);
int dts_should_checkpoint(int, const char* const*, int, const char* const*, const double*, double, int);
double dts_update_round_time(double, long long, long long);
}

#define CHECK(c)                                                     \
  do {                                                               \
    if (!(c)) {                                                      \
      std::fprintf(stderr, "CHECK failed %s:%d: %s\n", __FILE__, __LINE__, #c); \
      std::exit(1);                                                  \
    }                                                                \
  } while (0)

// ───────────────────────────── http ─────────────────────────────
static std::atomic<long long> g_handled{0};

static void echo_handler(void*, const char* method, const char* path, const char*, long long body_len, void* resp) {
  g_handled.fetch_add(1);
  std::string out = std::string(method) + " " + path + " " + std::to_string(body_len);
  dtr_http_respond(resp, 200, "text/plain", out.data(), (long long)out.size());
}

static int connect_to(int port) {
  int fd = ::socket(AF_INET, SOCK_STREAM, 0);
  sockaddr_in a{};
  a.sin_family = AF_INET;
  a.sin_port = htons((uint16_t)port);
  inet_pton(AF_INET, "127.0.0.1", &a.sin_addr);
  CHECK(::connect(fd, (sockaddr*)&a, sizeof a) == 0);
  return fd;
}

static bool send_all(int fd, const std::string& s) {
  size_t off = 0;
  while (off < s.size()) {
    ssize_t w = ::send(fd, s.data() + off, s.size() - off, MSG_NOSIGNAL);
    if (w <= 0) return false;
    off += (size_t)w;
  }
  return true;
}

// Reads one HTTP response (headers + Content-Length body); returns status and fills body.
static int read_response(int fd, std::string& pending, std::string& body) {
  for (;;) {
    size_t he = pending.find("\r\n\r\n");
    if (he != std::string::npos) {
      size_t cl_pos = pending.find("Content-Length:");
      if (cl_pos == std::string::npos || cl_pos > he) cl_pos = pending.find("content-length:");
      CHECK(cl_pos != std::string::npos && cl_pos < he);
      long long cl = std::atoll(pending.c_str() + cl_pos + 15);
      if ((long long)(pending.size() - he - 4) >= cl) {
        int status = std::atoi(pending.c_str() + 9);
        body = pending.substr(he + 4, (size_t)cl);
        pending.erase(0, he + 4 + (size_t)cl);
        return status;
      }
    }
    char buf[8192];
    ssize_t r = ::recv(fd, buf, sizeof buf, 0);
    if (r <= 0) return -1;
    pending.append(buf, (size_t)r);
  }
}

static void test_http() {
  void* srv = dtr_http_start("127.0.0.1", 0, 4, 1 << 20, echo_handler, nullptr);
  CHECK(srv != nullptr);
  const int port = dtr_http_port(srv);
  const int nclients = 8, nreq = 40;
  std::atomic<int> ok{0};
  std::vector<std::thread> cl;
  for (int c = 0; c < nclients; ++c) {
    cl.emplace_back([&, c] {
      int fd = connect_to(port);
      std::string pending, body;
      for (int i = 0; i < nreq; ++i) {
        const size_t len = (size_t)((c * 131 + i * 977) % 20000);
        std::string req = "POST /delta/" + std::to_string(c) + " HTTP/1.1\r\nHost: x\r\nContent-Length: " +
                          std::to_string(len) + "\r\n\r\n" + std::string(len, 'a' + (char)(i % 26));
        CHECK(send_all(fd, req));
        CHECK(read_response(fd, pending, body) == 200);
        CHECK(body == "POST /delta/" + std::to_string(c) + " " + std::to_string(len));
        ok.fetch_add(1);
      }
      ::close(fd);
    });
  }
  for (auto& t : cl) t.join();
  CHECK(ok.load() == nclients * nreq);
  // malformed request line and an oversized body: the server answers or closes, and keeps serving
  {
    int fd = connect_to(port);
    send_all(fd, "GARBAGE\r\n\r\n");
    std::string pending, body;
    read_response(fd, pending, body);
    ::close(fd);
    fd = connect_to(port);
    send_all(fd, "POST /x HTTP/1.1\r\nContent-Length: 99999999\r\n\r\n");
    read_response(fd, pending, body);
    ::close(fd);
    fd = connect_to(port);
    pending.clear();
    CHECK(send_all(fd, "GET /health HTTP/1.1\r\nContent-Length: 0\r\n\r\n"));
    CHECK(read_response(fd, pending, body) == 200);
    ::close(fd);
  }
  CHECK(dtr_http_served(srv) >= nclients * nreq);
  dtr_http_stop(srv);
}

// ───────────────────────────── codecs ─────────────────────────────
static void test_codecs() {
  // safetensors round trip of two tensors (names are written sorted)
  std::vector<float> a(6), b(5);
  for (int i = 0; i < 6; ++i) a[i] = 0.5f * (float)i - 1.0f;
  for (int i = 0; i < 5; ++i) b[i] = (float)(i * i);
  const char* names[2] = {"z.weight", "a.bias"};
  int ndims[2] = {2, 1};
  long long dims[3] = {2, 3, 5};
  const float* data[2] = {a.data(), b.data()};
  void* blob = nullptr;
  CHECK(dtr_st_save(nullptr, 2, names, ndims, dims, data, "{\"format\":\"pt\"}", &blob) == 0);
  CHECK(blob != nullptr && dtr_blob_size(blob) > 0);
  void* st = dtr_st_open_bytes(dtr_blob_data(blob), dtr_blob_size(blob));
  CHECK(st != nullptr && dtr_st_count(st) == 2);
  for (int i = 0; i < 2; ++i) {
    std::vector<float> back(8, -7.f);
    const bool isa = std::strcmp(dtr_st_name(st, i), "z.weight") == 0;
    const long long n = dtr_st_read_f32(st, i, back.data(), 8);
    CHECK(n == (isa ? 6 : 5));
    for (long long k = 0; k < n; ++k) CHECK(back[k] == (isa ? a[k] : b[k]));
  }
  dtr_st_close(st);
  dtr_blob_free(blob);

  // DTZ1: int8 + block scales, and fp32 values
  const long long total = 1000, count = 7;
  int idx[count] = {1, 5, 6, 100, 512, 513, 999};
  signed char q[count] = {1, -2, 3, -127, 127, 0, 64};
  float scales[1] = {0.25f};
  float vals[count] = {1.f, -2.f, 3.f, -4.f, 5.f, 6.f, -7.f};
  for (int quant = 0; quant < 2; ++quant) {
    void* enc = quant ? dtr_dtz_encode(total, count, idx, q, scales, nullptr, 256, 0)
                      : dtr_dtz_encode(total, count, idx, nullptr, nullptr, vals, 0, 0);
    CHECK(enc != nullptr);
    void* dec = dtr_dtz_decode_dense(dtr_blob_data(enc), dtr_blob_size(enc));
    CHECK(dec != nullptr && dtr_blob_size(dec) == total * 4);
    const float* d = static_cast<const float*>(dtr_blob_data(dec));
    for (long long k = 0; k < count; ++k) CHECK(d[idx[k]] == (quant ? (float)q[k] * scales[0] : vals[k]));
    CHECK(d[0] == 0.f && d[2] == 0.f);
    dtr_blob_free(dec);
    dtr_blob_free(enc);
  }

  // hashing / shard assignment are pure functions
  const char msg[] = "distrain";
  CHECK(dtr_siphash13(msg, 8) == dtr_siphash13(msg, 8));
  CHECK(dtr_splitmix64(1) != dtr_splitmix64(2));
  long long s1[16], s2[16];
  const long long n1 = dtr_shard_assignment("node-00", 3, 100, 16, s1);
  const long long n2 = dtr_shard_assignment("node-00", 3, 100, 16, s2);
  CHECK(n1 > 0 && n1 == n2);
  for (long long i = 0; i < n1; ++i) CHECK(s1[i] == s2[i] && s1[i] >= 0 && s1[i] < 100);

  if (dtr_zstd_available()) {
    std::string text(100000, 'x');
    for (size_t i = 0; i < text.size(); i += 97) text[i] = (char)('a' + i % 23);
    void* z = dtr_zstd_compress(text.data(), (long long)text.size(), 3);
    CHECK(z != nullptr && dtr_blob_size(z) < (long long)text.size());
    void* u = dtr_zstd_decompress(dtr_blob_data(z), dtr_blob_size(z));
    CHECK(u != nullptr && dtr_blob_size(u) == (long long)text.size());
    CHECK(std::memcmp(dtr_blob_data(u), text.data(), text.size()) == 0);
    dtr_blob_free(u);
    dtr_blob_free(z);
  }
}

// ───────────────────────────── loader ─────────────────────────────
static void test_loader(const std::string& dir) {
  const int nshard = 3;
  const size_t per = 5000;
  std::string paths;
  uint16_t tok = 0;
  for (int s = 0; s < nshard; ++s) {
    std::string p = dir + "/shard_" + std::to_string(s) + ".bin";
    std::vector<uint16_t> v(per);
    for (auto& x : v) x = tok++;
    FILE* f = std::fopen(p.c_str(), "wb");
    CHECK(f != nullptr);
    CHECK(std::fwrite(v.data(), 2, per, f) == per);
    std::fclose(f);
    paths += p + "\n";
  }
  const long long seq = 64, batch = 8;
  void* L = dtr_loader_open(paths.c_str(), seq, batch, 2);
  CHECK(L != nullptr);
  // synchronous: tokens come out in file order, widened to int32, wrapping at the end
  std::vector<int32_t> out((size_t)(seq * batch));
  long long expect = 0;
  const long long total = nshard * (long long)per;
  for (int it = 0; it < 40; ++it) {
    CHECK(dtr_loader_next(L, out.data(), batch) == 0);
    for (long long k = 0; k < seq * batch; ++k) {
      CHECK(out[(size_t)k] == (int32_t)(expect % total));
      ++expect;
    }
  }
  // prefetch thread + consumer
  dtr_loader_reset(L);
  std::vector<std::vector<int32_t>> bufs(3, std::vector<int32_t>((size_t)(seq * batch)));
  int32_t* ptrs[3] = {bufs[0].data(), bufs[1].data(), bufs[2].data()};
  CHECK(dtr_loader_start_prefetch(L, ptrs, 3) == 0);
  expect = 0;
  for (int it = 0; it < 200; ++it) {
    const int s = dtr_loader_acquire(L, 5000);
    CHECK(s >= 0 && s < 3);
    for (long long k = 0; k < seq * batch; k += 61) CHECK(bufs[(size_t)s][(size_t)k] == (int32_t)((expect + k) % total));
    expect += seq * batch;
    dtr_loader_release(L, s);
  }
  dtr_loader_close(L);
}

// ───────────────────────────── scheduler ─────────────────────────────
static void test_scheduler() {
  const char* nodes[2] = {"a", "b"};
  long long seqs[2] = {3, 1};
  double w = 0;
  char why[128];
  CHECK(dts_accept_push(10, 8, 5, 2, nodes, seqs, "c", 1, 1000.0, 0.9, &w, why, sizeof why) == 1);
  CHECK(std::fabs(w - 1000.0 * 0.81) < 1e-9);
  CHECK(dts_accept_push(10, 2, 5, 2, nodes, seqs, "c", 1, 1000.0, 0.9, &w, why, sizeof why) == 0);
  CHECK(std::strncmp(why, "Too stale", 9) == 0);
  CHECK(dts_accept_push(10, 10, 5, 2, nodes, seqs, "a", 3, 1000.0, 0.9, &w, why, 8) == 0);  // truncated reason
  CHECK(std::strlen(why) < 8);
  const char* active[3] = {"a", "b", "c"};
  double times[3] = {100.0, std::nan(""), 40.0};
  CHECK(dts_should_checkpoint(0, nodes, 3, active, times, 1000.0, 0) == 0);
  CHECK(dts_should_checkpoint(2, nodes, 3, active, times, 10.0, 0) == 0);   // patience 120 s not elapsed
  CHECK(dts_should_checkpoint(2, nodes, 3, active, times, 120.7, 0) == 1);
  CHECK(dts_should_checkpoint(2, nodes, 2, active, times, 0.0, 0) == 1);    // every active node contributed
  CHECK(dts_update_round_time(std::nan(""), -1, 100) != dts_update_round_time(std::nan(""), -1, 100));
  CHECK(dts_update_round_time(std::nan(""), 100, 200) == 100.0);
}

int main(int argc, char** argv) {
  const std::string dir = argc > 1 ? argv[1] : "/tmp";
  test_codecs();
  test_scheduler();
  test_loader(dir);
  test_http();
  std::printf("runtime selftest ok\n");
  return 0;
}
