// Host runtime of the framework (no CUDA): checkpoint file IO and the token data pipeline.
#pragma once
#include <stddef.h>
#include <stdint.h>

#include <condition_variable>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace mxrt {

// ------------------------------------------------------------------------------------------ io
uint32_t crc32c(const void* data, size_t n, uint32_t seed);
// Returns the CRC-32C of every `piece`-byte piece of every file.
std::vector<std::vector<uint32_t>> write_files(const std::vector<std::string>& paths,
                                               const std::vector<const void*>& bufs,
                                               const std::vector<size_t>& sizes, int threads, bool do_fsync,
                                               size_t piece);
std::vector<std::vector<uint32_t>> read_files(const std::vector<std::string>& paths, const std::vector<void*>& bufs,
                                              const std::vector<size_t>& sizes, int threads, size_t piece);

// ---------------------------------------------------------------------------------------- data
uint64_t mix64(uint64_t x);

// Keyed bijection of [0, n): a 4-round balanced Feistel network over the next power of two,
// with cycle walking (Black & Rogaway, "Ciphers with Arbitrary Finite Domains", 2002).
class Permutation {
 public:
  Permutation(uint64_t n, uint64_t key);
  uint64_t operator()(uint64_t i) const;
  uint64_t size() const { return n_; }

 private:
  uint64_t n_, key_;
  int half_bits_;
  uint64_t half_mask_;
};

// One training example: tokens, segment ids (packed documents) and next-token loss weights.
struct ExampleOut {
  int32_t* tokens;
  int32_t* segments;
  float* loss_weight;
};

class Dataset {
 public:
  virtual ~Dataset() = default;
  virtual uint64_t size() const = 0;  // examples per epoch
  virtual int seq_len() const = 0;
  // Fill example `idx` (idx may exceed size(): datasets wrap into later epochs).
  virtual void fill(uint64_t idx, const ExampleOut& out) const = 0;
};

// Deterministic random ids in [1, vocab); segments of doc_len tokens.
class SyntheticDataset : public Dataset {
 public:
  SyntheticDataset(int seq_len, int vocab, int doc_len, uint64_t seed)
      : S_(seq_len), V_(vocab), doc_len_(doc_len > 0 ? doc_len : seq_len), seed_(seed) {}
  uint64_t size() const override { return uint64_t(1) << 62; }
  int seq_len() const override { return S_; }
  void fill(uint64_t idx, const ExampleOut& out) const override;

 private:
  int S_, V_, doc_len_;
  uint64_t seed_;
};

// Memory-mapped token cache: shards of little-endian uint32 token ids with uint64 document end
// offsets, read as one concatenated stream chopped into seq_len windows.
class TokenSeqDataset : public Dataset {
 public:
  TokenSeqDataset(const std::vector<std::string>& token_files, const std::vector<std::string>& doc_files,
                  int seq_len, uint64_t seed, bool shuffle,
                  const std::vector<std::string>& mask_files = std::vector<std::string>());
  ~TokenSeqDataset() override;
  uint64_t size() const override { return n_seq_; }
  int seq_len() const override { return S_; }
  void fill(uint64_t idx, const ExampleOut& out) const override;
  uint64_t total_tokens() const { return total_; }

 private:
  struct Shard {
    const uint32_t* tok = nullptr;
    uint64_t ntok = 0;
    const uint64_t* ends = nullptr;
    uint64_t ndocs = 0;
    void* map_tok = nullptr;
    size_t map_tok_len = 0;
    void* map_ends = nullptr;
    size_t map_ends_len = 0;
    const uint8_t* mask = nullptr;  // optional per-token loss mask (1 = train on this token)
    void* map_mask = nullptr;
    size_t map_mask_len = 0;
  };
  std::vector<Shard> shards_;
  std::vector<uint64_t> base_;  // first global token of each shard
  uint64_t total_ = 0, n_seq_ = 0;
  int S_;
  uint64_t seed_;
  bool shuffle_;
  // document id (global, monotone) of global token position g, and the end of that document
  void locate(uint64_t g, uint64_t& doc, uint64_t& doc_end) const;
};

enum class StopStrategy { kRestart = 0, kFirstExhausted = 1 };

// Weighted mixture with block-deterministic sampling: each block of `block_size` consecutive
// examples holds round(w_c * block_size) examples of component c (largest remainder), in an order
// given by a per-block keyed permutation. Weight stages switch at example indices.
class MixtureDataset : public Dataset {
 public:
  MixtureDataset(std::vector<std::shared_ptr<Dataset>> comps, std::vector<uint64_t> stage_starts,
                 std::vector<std::vector<double>> stage_weights, uint64_t block_size, uint64_t seed,
                 StopStrategy stop);
  uint64_t size() const override { return uint64_t(1) << 62; }
  int seq_len() const override { return comps_[0]->seq_len(); }
  void fill(uint64_t idx, const ExampleOut& out) const override;
  // (component, component-local index) of mixture example idx
  void resolve(uint64_t idx, int& comp, uint64_t& local) const;

 private:
  std::vector<std::shared_ptr<Dataset>> comps_;
  std::vector<uint64_t> stage_block_;  // first block of each stage
  std::vector<std::vector<uint64_t>> stage_counts_;  // per stage: examples per component per block
  uint64_t block_;
  uint64_t seed_;
  StopStrategy stop_;
};

void fill_batch(const Dataset& ds, uint64_t first, int count, int32_t* tokens, int32_t* segments, float* lw,
                int threads);

// Background batch producer over a ring of caller-owned (pinned) host buffers.
class Prefetcher {
 public:
  Prefetcher(std::shared_ptr<Dataset> ds, int local_batch, int global_batch, int rank, uint64_t start_step,
             std::vector<int32_t*> tok, std::vector<int32_t*> seg, std::vector<float*> lw, int threads);
  ~Prefetcher();
  // Blocks (bounded by timeout_s) until the next step's batch is ready; returns its slot.
  int next(double timeout_s, uint64_t& step);
  void release(int slot);

 private:
  void run();
  std::shared_ptr<Dataset> ds_;
  int lb_, gb_, rank_, threads_;
  std::vector<int32_t*> tok_, seg_;
  std::vector<float*> lw_;
  int depth_;
  std::vector<int> state_;  // 0 free, 1 filling, 2 ready, 3 handed out
  std::vector<uint64_t> slot_step_;
  uint64_t produce_step_, consume_step_;
  std::string error_;
  uint64_t error_step_ = 0;
  bool stop_ = false;
  std::mutex mu_;
  std::condition_variable cv_;
  std::thread worker_;
};

}  // namespace mxrt
