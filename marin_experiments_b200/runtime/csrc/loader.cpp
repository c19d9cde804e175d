// Token data pipeline: synthetic / memory-mapped token caches, weighted block mixtures, batch
// assembly with packed-document segment ids and next-token loss weights, and a background
// prefetcher that fills a ring of pinned host buffers.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <numeric>
#include <stdexcept>

#include "rt.h"

namespace mxrt {

// SplitMix64 finaliser (Steele, Lea & Flood, "Fast splittable pseudorandom number generators",
// OOPSLA 2014).
uint64_t mix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

Permutation::Permutation(uint64_t n, uint64_t key) : n_(n), key_(key) {
  int bits = 1;
  while (bits < 64 && (uint64_t(1) << bits) < n) ++bits;
  if (bits & 1) ++bits;
  half_bits_ = bits / 2;
  half_mask_ = (uint64_t(1) << half_bits_) - 1;
}

uint64_t Permutation::operator()(uint64_t i) const {
  if (n_ <= 1) return 0;
  uint64_t x = i;
  do {
    uint64_t l = x >> half_bits_, r = x & half_mask_;
    for (int round = 0; round < 4; ++round) {
      const uint64_t f = mix64(key_ ^ (uint64_t(round) << 56) ^ r) & half_mask_;
      const uint64_t nl = r;
      r = l ^ f;
      l = nl;
    }
    x = (l << half_bits_) | r;
  } while (x >= n_);  // cycle walking: the domain is the next even power of two >= n
  return x;
}

// ------------------------------------------------------------------------------- synthetic
void SyntheticDataset::fill(uint64_t idx, const ExampleOut& out) const {
  const uint64_t base = mix64(seed_ * 0x100000001B3ull ^ mix64(idx));
  for (int p = 0; p < S_; ++p) {
    const uint64_t r = mix64(base + (uint64_t)p);
    out.tokens[p] = 1 + (int32_t)(r % (uint64_t)(V_ - 1));
    out.segments[p] = p / doc_len_;
  }
  for (int p = 0; p < S_; ++p)
    out.loss_weight[p] = (p + 1 < S_ && out.segments[p + 1] == out.segments[p]) ? 1.f : 0.f;
}

// ------------------------------------------------------------------------------ token cache
namespace {
void* map_file(const std::string& path, size_t& len) {
  int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) throw std::runtime_error("cannot open " + path);
  struct stat st;
  if (::fstat(fd, &st) != 0) {
    ::close(fd);
    throw std::runtime_error("cannot stat " + path);
  }
  len = (size_t)st.st_size;
  void* p = nullptr;
  if (len > 0) {
    p = ::mmap(nullptr, len, PROT_READ, MAP_SHARED, fd, 0);
    if (p == MAP_FAILED) {
      ::close(fd);
      throw std::runtime_error("mmap failed for " + path);
    }
    ::madvise(p, len, MADV_RANDOM);
  }
  ::close(fd);
  return p;
}
}  // namespace

TokenSeqDataset::TokenSeqDataset(const std::vector<std::string>& token_files,
                                 const std::vector<std::string>& doc_files, int seq_len, uint64_t seed, bool shuffle,
                                 const std::vector<std::string>& mask_files)
    : S_(seq_len), seed_(seed), shuffle_(shuffle) {
  if (token_files.size() != doc_files.size() || token_files.empty())
    throw std::runtime_error("token cache needs one document file per token file");
  if (!mask_files.empty() && mask_files.size() != token_files.size())
    throw std::runtime_error("token cache needs one mask file per token file (or none)");
  for (size_t i = 0; i < token_files.size(); ++i) {
    Shard s;
    s.map_tok = map_file(token_files[i], s.map_tok_len);
    s.tok = static_cast<const uint32_t*>(s.map_tok);
    s.ntok = s.map_tok_len / 4;
    s.map_ends = map_file(doc_files[i], s.map_ends_len);
    s.ends = static_cast<const uint64_t*>(s.map_ends);
    s.ndocs = s.map_ends_len / 8;
    if (s.ndocs == 0 || s.ends[s.ndocs - 1] != s.ntok)
      throw std::runtime_error("document offsets of " + doc_files[i] + " do not end at the token count");
    if (!mask_files.empty()) {
      s.map_mask = map_file(mask_files[i], s.map_mask_len);
      s.mask = static_cast<const uint8_t*>(s.map_mask);
      if (s.map_mask_len != s.ntok) throw std::runtime_error("mask file " + mask_files[i] + " length != token count");
    }
    base_.push_back(total_);
    total_ += s.ntok;
    shards_.push_back(s);
  }
  n_seq_ = total_ / (uint64_t)S_;
  if (n_seq_ == 0) throw std::runtime_error("token cache shorter than one sequence");
}

TokenSeqDataset::~TokenSeqDataset() {
  for (auto& s : shards_) {
    if (s.map_tok) ::munmap(s.map_tok, s.map_tok_len);
    if (s.map_ends) ::munmap(s.map_ends, s.map_ends_len);
    if (s.map_mask) ::munmap(s.map_mask, s.map_mask_len);
  }
}

void TokenSeqDataset::locate(uint64_t g, uint64_t& doc, uint64_t& doc_end) const {
  const size_t si = (size_t)(std::upper_bound(base_.begin(), base_.end(), g) - base_.begin()) - 1;
  const Shard& s = shards_[si];
  const uint64_t local = g - base_[si];
  const uint64_t* it = std::upper_bound(s.ends, s.ends + s.ndocs, local);
  const uint64_t di = (uint64_t)(it - s.ends);
  uint64_t docs_before = 0;
  for (size_t k = 0; k < si; ++k) docs_before += shards_[k].ndocs;
  doc = docs_before + di;
  doc_end = base_[si] + s.ends[di];
}

void TokenSeqDataset::fill(uint64_t idx, const ExampleOut& out) const {
  const uint64_t epoch = idx / n_seq_, i = idx % n_seq_;
  uint64_t seq = i;
  if (shuffle_) seq = Permutation(n_seq_, mix64(seed_ ^ mix64(epoch + 0x5EEDull)))(i);
  uint64_t g = seq * (uint64_t)S_;
  uint64_t doc, doc_end;
  locate(g, doc, doc_end);
  size_t si = (size_t)(std::upper_bound(base_.begin(), base_.end(), g) - base_.begin()) - 1;
  int seg = 0;
  for (int p = 0; p < S_; ++p, ++g) {
    while (g >= doc_end) {  // crossed into the next document
      ++seg;
      locate(g, doc, doc_end);
    }
    while (si + 1 < base_.size() && g >= base_[si + 1]) ++si;
    out.tokens[p] = (int32_t)shards_[si].tok[g - base_[si]];
    out.segments[p] = seg;
    // position p predicts token p + 1: stash that token's mask in loss_weight[p - 1]
    if (p > 0) out.loss_weight[p - 1] = shards_[si].mask ? (float)shards_[si].mask[g - base_[si]] : 1.f;
  }
  out.loss_weight[S_ - 1] = 0.f;
  for (int p = 0; p + 1 < S_; ++p)
    if (out.segments[p + 1] != out.segments[p]) out.loss_weight[p] = 0.f;
}

// --------------------------------------------------------------------------------- mixture
MixtureDataset::MixtureDataset(std::vector<std::shared_ptr<Dataset>> comps, std::vector<uint64_t> stage_starts,
                               std::vector<std::vector<double>> stage_weights, uint64_t block_size, uint64_t seed,
                               StopStrategy stop)
    : comps_(std::move(comps)), block_(block_size), seed_(seed), stop_(stop) {
  if (comps_.empty() || block_ == 0) throw std::runtime_error("mixture needs components and a block size");
  if (stage_starts.empty() || stage_starts[0] != 0 || stage_starts.size() != stage_weights.size())
    throw std::runtime_error("mixture stages must start at example 0");
  for (auto& c : comps_)
    if (c->seq_len() != comps_[0]->seq_len()) throw std::runtime_error("mixture components differ in seq_len");
  for (size_t s = 0; s < stage_starts.size(); ++s) {
    if (stage_starts[s] % block_) throw std::runtime_error("mixture stage starts must be multiples of the block size");
    if (s && stage_starts[s] <= stage_starts[s - 1]) throw std::runtime_error("mixture stages must increase");
    const auto& w = stage_weights[s];
    if (w.size() != comps_.size()) throw std::runtime_error("one weight per component");
    double tot = 0;
    for (double x : w) {
      if (x < 0) throw std::runtime_error("negative mixture weight");
      tot += x;
    }
    if (tot <= 0) throw std::runtime_error("mixture weights sum to zero");
    // largest remainder apportionment of block_ examples
    std::vector<uint64_t> cnt(w.size());
    std::vector<std::pair<double, size_t>> rem;
    uint64_t used = 0;
    for (size_t c = 0; c < w.size(); ++c) {
      const double q = w[c] / tot * (double)block_;
      cnt[c] = (uint64_t)std::floor(q);
      used += cnt[c];
      rem.push_back({q - std::floor(q), c});
    }
    std::stable_sort(rem.begin(), rem.end(), [](auto& a, auto& b) { return a.first > b.first; });
    for (size_t k = 0; used < block_; ++k, ++used) cnt[rem[k % rem.size()].second]++;
    stage_block_.push_back(stage_starts[s] / block_);
    stage_counts_.push_back(cnt);
  }
}

void MixtureDataset::resolve(uint64_t idx, int& comp, uint64_t& local) const {
  const uint64_t b = idx / block_, j = idx % block_;
  size_t st = 0;
  while (st + 1 < stage_block_.size() && stage_block_[st + 1] <= b) ++st;
  const auto& cnt = stage_counts_[st];
  const uint64_t q = Permutation(block_, mix64(seed_ ^ mix64(b + 0xB10Cull)))(j);
  uint64_t acc = 0;
  size_t c = 0;
  while (q >= acc + cnt[c]) acc += cnt[c++];
  // examples of component c in all earlier blocks
  uint64_t before = 0;
  for (size_t s = 0; s <= st; ++s) {
    const uint64_t b0 = stage_block_[s];
    const uint64_t b1 = s == st ? b : stage_block_[s + 1];
    before += (b1 - b0) * stage_counts_[s][c];
  }
  comp = (int)c;
  local = before + (q - acc);
}

void MixtureDataset::fill(uint64_t idx, const ExampleOut& out) const {
  int c;
  uint64_t local;
  resolve(idx, c, local);
  if (stop_ == StopStrategy::kFirstExhausted && local >= comps_[c]->size())
    throw std::out_of_range("mixture component exhausted");
  comps_[c]->fill(local, out);
}

void fill_batch(const Dataset& ds, uint64_t first, int count, int32_t* tokens, int32_t* segments, float* lw,
                int threads) {
  const int S = ds.seq_len();
  auto one = [&](int i) {
    ExampleOut o{tokens + (size_t)i * S, segments + (size_t)i * S, lw + (size_t)i * S};
    ds.fill(first + (uint64_t)i, o);
  };
  if (threads <= 1 || count <= 1) {
    for (int i = 0; i < count; ++i) one(i);
    return;
  }
  std::atomic<int> next{0};
  std::string err;
  std::mutex emu;
  std::vector<std::thread> pool;
  for (int t = 0; t < std::min(threads, count); ++t)
    pool.emplace_back([&] {
      for (int i = next++; i < count; i = next++) {
        try {
          one(i);
        } catch (const std::exception& e) {
          std::lock_guard<std::mutex> g(emu);
          if (err.empty()) err = e.what();
        }
      }
    });
  for (auto& th : pool) th.join();
  if (!err.empty()) {
    if (err.find("exhausted") != std::string::npos) throw std::out_of_range(err);
    throw std::runtime_error(err);
  }
}

// ------------------------------------------------------------------------------- prefetcher
Prefetcher::Prefetcher(std::shared_ptr<Dataset> ds, int local_batch, int global_batch, int rank,
                       uint64_t start_step, std::vector<int32_t*> tok, std::vector<int32_t*> seg,
                       std::vector<float*> lw, int threads)
    : ds_(std::move(ds)), lb_(local_batch), gb_(global_batch), rank_(rank), threads_(threads), tok_(std::move(tok)),
      seg_(std::move(seg)), lw_(std::move(lw)) {
  depth_ = (int)tok_.size();
  if (depth_ < 1 || seg_.size() != tok_.size() || lw_.size() != tok_.size())
    throw std::runtime_error("prefetcher needs matching slot buffers");
  state_.assign(depth_, 0);
  slot_step_.assign(depth_, 0);
  produce_step_ = consume_step_ = start_step;
  worker_ = std::thread([this] { run(); });
}

Prefetcher::~Prefetcher() {
  {
    std::lock_guard<std::mutex> g(mu_);
    stop_ = true;
  }
  cv_.notify_all();
  if (worker_.joinable()) worker_.join();
}

void Prefetcher::run() {
  for (;;) {
    int slot;
    uint64_t step;
    {
      std::unique_lock<std::mutex> g(mu_);
      slot = (int)(produce_step_ % depth_);
      cv_.wait(g, [&] { return stop_ || state_[slot] == 0; });
      if (stop_ || !error_.empty()) return;
      state_[slot] = 1;
      step = produce_step_++;
    }
    std::string err;
    try {
      const uint64_t first = step * (uint64_t)gb_ + (uint64_t)rank_ * (uint64_t)lb_;
      fill_batch(*ds_, first, lb_, tok_[slot], seg_[slot], lw_[slot], threads_);
    } catch (const std::exception& e) {
      err = e.what();
    }
    {
      std::lock_guard<std::mutex> g(mu_);
      slot_step_[slot] = step;
      state_[slot] = 2;
      if (!err.empty()) {
        error_ = err;
        error_step_ = step;
      }
    }
    cv_.notify_all();
    if (!err.empty()) return;
  }
}

int Prefetcher::next(double timeout_s, uint64_t& step) {
  std::unique_lock<std::mutex> g(mu_);
  const int slot = (int)(consume_step_ % depth_);
  auto failed = [&] { return !error_.empty() && consume_step_ >= error_step_; };
  const bool ok = cv_.wait_for(g, std::chrono::duration<double>(timeout_s),
                               [&] { return failed() || state_[slot] == 2; });
  if (failed()) {
    if (error_.find("exhausted") != std::string::npos) throw std::out_of_range(error_);
    throw std::runtime_error(error_);
  }
  if (!ok) throw std::runtime_error("data prefetcher timed out");
  state_[slot] = 3;
  step = consume_step_++;
  return slot;
}

void Prefetcher::release(int slot) {
  {
    std::lock_guard<std::mutex> g(mu_);
    if (slot >= 0 && slot < depth_ && state_[slot] == 3) state_[slot] = 0;
  }
  cv_.notify_all();
}

}  // namespace mxrt
