// Parallel file IO for checkpoints.
//
// A checkpoint is a set of (path, host buffer) pairs. Every buffer is cut into pieces of
// kPiece bytes; a pool of threads writes (pwrite) or reads (pread) the pieces of all files
// concurrently and computes a CRC-32C of each piece, so one 10 GB flat buffer and a thousand
// small leaves both spread over every thread. The CRC uses the SSE4.2 crc32 instruction when the
// CPU has it, else a byte-wise table over the Castagnoli polynomial 0x82F63B78 (reflected).
#include "rt.h"

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <atomic>
#include <cerrno>
#include <cstring>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace mxrt {

namespace {

uint32_t g_table[256];
bool g_table_ready = false;
bool g_hw = false;

void init_crc() {
  if (g_table_ready) return;
  for (uint32_t i = 0; i < 256; ++i) {
    uint32_t c = i;
    for (int k = 0; k < 8; ++k) c = (c & 1) ? (c >> 1) ^ 0x82F63B78u : (c >> 1);
    g_table[i] = c;
  }
#if defined(__x86_64__)
  g_hw = __builtin_cpu_supports("sse4.2");
#endif
  g_table_ready = true;
}

uint32_t crc_sw(uint32_t crc, const uint8_t* p, size_t n) {
  for (size_t i = 0; i < n; ++i) crc = g_table[(crc ^ p[i]) & 0xFF] ^ (crc >> 8);
  return crc;
}

#if defined(__x86_64__)
__attribute__((target("sse4.2"))) uint32_t crc_hw(uint32_t crc, const uint8_t* p, size_t n) {
  uint64_t c = crc;
  while (n >= 8) {
    uint64_t v;
    std::memcpy(&v, p, 8);
    c = __builtin_ia32_crc32di(c, v);
    p += 8;
    n -= 8;
  }
  uint32_t c32 = (uint32_t)c;
  while (n--) c32 = __builtin_ia32_crc32qi(c32, *p++);
  return c32;
}
#endif

struct Piece {
  int file;
  size_t off, len;
};

std::vector<Piece> make_pieces(const std::vector<size_t>& sizes, size_t piece) {
  std::vector<Piece> out;
  for (size_t f = 0; f < sizes.size(); ++f) {
    if (sizes[f] == 0) continue;
    for (size_t o = 0; o < sizes[f]; o += piece) out.push_back({(int)f, o, std::min(piece, sizes[f] - o)});
  }
  return out;
}

template <class Fn>
void run_pool(size_t n_items, int threads, Fn fn) {
  if (threads <= 1 || n_items <= 1) {
    for (size_t i = 0; i < n_items; ++i) fn(i);
    return;
  }
  std::atomic<size_t> next{0};
  std::vector<std::thread> pool;
  const int nt = (int)std::min<size_t>(threads, n_items);
  for (int t = 0; t < nt; ++t)
    pool.emplace_back([&] {
      for (size_t i = next++; i < n_items; i = next++) fn(i);
    });
  for (auto& th : pool) th.join();
}

}  // namespace

uint32_t crc32c(const void* data, size_t n, uint32_t seed) {
  init_crc();
  uint32_t c = ~seed;
#if defined(__x86_64__)
  if (g_hw) return ~crc_hw(c, static_cast<const uint8_t*>(data), n);
#endif
  return ~crc_sw(c, static_cast<const uint8_t*>(data), n);
}

std::vector<std::vector<uint32_t>> write_files(const std::vector<std::string>& paths,
                                               const std::vector<const void*>& bufs,
                                               const std::vector<size_t>& sizes, int threads, bool do_fsync,
                                               size_t piece) {
  init_crc();
  const size_t nf = paths.size();
  std::vector<int> fds(nf, -1);
  for (size_t f = 0; f < nf; ++f) {
    fds[f] = ::open(paths[f].c_str(), O_WRONLY | O_CREAT | O_TRUNC, 0644);
    if (fds[f] < 0) {
      for (size_t g = 0; g < f; ++g) ::close(fds[g]);
      throw std::runtime_error("open for write failed: " + paths[f] + ": " + std::strerror(errno));
    }
    if (sizes[f] && ::ftruncate(fds[f], (off_t)sizes[f]) != 0) {
      for (size_t g = 0; g <= f; ++g) ::close(fds[g]);
      throw std::runtime_error("ftruncate failed: " + paths[f]);
    }
  }
  auto pieces = make_pieces(sizes, piece);
  std::vector<std::vector<uint32_t>> crcs(nf);
  for (size_t f = 0; f < nf; ++f) crcs[f].resize((sizes[f] + piece - 1) / piece);
  std::atomic<int> failed{0};
  run_pool(pieces.size(), threads, [&](size_t i) {
    const Piece& pc = pieces[i];
    const uint8_t* src = static_cast<const uint8_t*>(bufs[pc.file]) + pc.off;
    size_t done = 0;
    while (done < pc.len) {
      ssize_t w = ::pwrite(fds[pc.file], src + done, pc.len - done, (off_t)(pc.off + done));
      if (w < 0 && errno == EINTR) continue;
      if (w <= 0) {
        failed = 1;
        return;
      }
      done += (size_t)w;
    }
    crcs[pc.file][pc.off / piece] = crc32c(src, pc.len, 0);
  });
  if (do_fsync) run_pool(nf, threads, [&](size_t f) { ::fsync(fds[f]); });
  for (int fd : fds) ::close(fd);
  if (failed) throw std::runtime_error("pwrite failed");
  return crcs;
}

std::vector<std::vector<uint32_t>> read_files(const std::vector<std::string>& paths, const std::vector<void*>& bufs,
                                              const std::vector<size_t>& sizes, int threads, size_t piece) {
  init_crc();
  const size_t nf = paths.size();
  std::vector<int> fds(nf, -1);
  for (size_t f = 0; f < nf; ++f) {
    fds[f] = ::open(paths[f].c_str(), O_RDONLY);
    struct stat st;
    if (fds[f] < 0 || ::fstat(fds[f], &st) != 0 || (size_t)st.st_size < sizes[f]) {
      for (size_t g = 0; g <= f; ++g)
        if (fds[g] >= 0) ::close(fds[g]);
      throw std::runtime_error("missing or short file: " + paths[f]);
    }
  }
  auto pieces = make_pieces(sizes, piece);
  std::vector<std::vector<uint32_t>> crcs(nf);
  for (size_t f = 0; f < nf; ++f) crcs[f].resize((sizes[f] + piece - 1) / piece);
  std::atomic<int> failed{0};
  run_pool(pieces.size(), threads, [&](size_t i) {
    const Piece& pc = pieces[i];
    uint8_t* dst = static_cast<uint8_t*>(bufs[pc.file]) + pc.off;
    size_t done = 0;
    while (done < pc.len) {
      ssize_t r = ::pread(fds[pc.file], dst + done, pc.len - done, (off_t)(pc.off + done));
      if (r < 0 && errno == EINTR) continue;
      if (r <= 0) {
        failed = 1;
        return;
      }
      done += (size_t)r;
    }
    crcs[pc.file][pc.off / piece] = crc32c(dst, pc.len, 0);
  });
  for (int fd : fds) ::close(fd);
  if (failed) throw std::runtime_error("pread failed");
  return crcs;
}

}  // namespace mxrt
