// Python bindings of the host runtime (checkpoint IO, data pipeline).
#include <torch/extension.h>

#include <stdexcept>

#include "rt.h"

namespace {

void check_host(const at::Tensor& t, const char* name) {
  TORCH_CHECK(!t.is_cuda(), name, " must be a host tensor");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

size_t nbytes(const at::Tensor& t) { return (size_t)t.numel() * t.element_size(); }

std::vector<std::vector<uint32_t>> write_files(const std::vector<std::string>& paths,
                                               const std::vector<at::Tensor>& bufs, int64_t threads, bool do_fsync,
                                               int64_t piece) {
  TORCH_CHECK(paths.size() == bufs.size(), "one buffer per path");
  std::vector<const void*> ptrs;
  std::vector<size_t> sizes;
  for (auto& b : bufs) {
    check_host(b, "buffer");
    ptrs.push_back(b.data_ptr());
    sizes.push_back(nbytes(b));
  }
  pybind11::gil_scoped_release nogil;
  return mxrt::write_files(paths, ptrs, sizes, (int)threads, do_fsync, (size_t)piece);
}

std::vector<std::vector<uint32_t>> read_files(const std::vector<std::string>& paths,
                                              const std::vector<at::Tensor>& bufs, int64_t threads, int64_t piece) {
  TORCH_CHECK(paths.size() == bufs.size(), "one buffer per path");
  std::vector<void*> ptrs;
  std::vector<size_t> sizes;
  for (auto& b : bufs) {
    check_host(b, "buffer");
    ptrs.push_back(b.data_ptr());
    sizes.push_back(nbytes(b));
  }
  pybind11::gil_scoped_release nogil;
  try {
    return mxrt::read_files(paths, ptrs, sizes, (int)threads, (size_t)piece);
  } catch (const std::runtime_error& e) {
    if (std::string(e.what()).rfind("missing", 0) == 0) {
      pybind11::gil_scoped_acquire gil;
      throw pybind11::value_error(std::string("FileNotFound: ") + e.what());
    }
    throw;
  }
}

uint32_t crc32c(const at::Tensor& t) {
  check_host(t, "buffer");
  return mxrt::crc32c(t.data_ptr(), nbytes(t), 0);
}

void check_batch(const mxrt::Dataset& ds, const at::Tensor& tok, const at::Tensor& seg, const at::Tensor& lw) {
  check_host(tok, "tokens");
  check_host(seg, "segment_ids");
  check_host(lw, "loss_weight");
  TORCH_CHECK(tok.scalar_type() == at::kInt && seg.scalar_type() == at::kInt && lw.scalar_type() == at::kFloat,
              "tokens/segment_ids int32, loss_weight float32");
  TORCH_CHECK(tok.dim() == 2 && tok.size(1) == ds.seq_len(), "tokens must be [batch, seq_len]");
  TORCH_CHECK(seg.sizes() == tok.sizes() && lw.sizes() == tok.sizes(), "batch buffers must match");
}

// Owns the slot tensors for as long as the worker thread can write into them: members are destroyed in
// reverse order, so the prefetcher (and its thread) goes first.
struct PyPrefetcher {
  std::vector<at::Tensor> keep;
  std::unique_ptr<mxrt::Prefetcher> pf;
};

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("write_files", &write_files, pybind11::arg("paths"), pybind11::arg("bufs"), pybind11::arg("threads") = 8,
        pybind11::arg("fsync") = false, pybind11::arg("piece") = 16 << 20);
  m.def("read_files", &read_files, pybind11::arg("paths"), pybind11::arg("bufs"), pybind11::arg("threads") = 8,
        pybind11::arg("piece") = 16 << 20);
  m.def("crc32c", &crc32c);

  pybind11::class_<mxrt::Dataset, std::shared_ptr<mxrt::Dataset>>(m, "Dataset")
      .def("size", &mxrt::Dataset::size)
      .def("seq_len", &mxrt::Dataset::seq_len)
      .def("fill_batch",
           [](const mxrt::Dataset& ds, uint64_t first, at::Tensor tok, at::Tensor seg, at::Tensor lw, int threads) {
             check_batch(ds, tok, seg, lw);
             pybind11::gil_scoped_release nogil;
             mxrt::fill_batch(ds, first, (int)tok.size(0), tok.data_ptr<int32_t>(), seg.data_ptr<int32_t>(),
                              lw.data_ptr<float>(), threads);
           },
           pybind11::arg("first"), pybind11::arg("tokens"), pybind11::arg("segment_ids"),
           pybind11::arg("loss_weight"), pybind11::arg("threads") = 4);
  pybind11::class_<mxrt::SyntheticDataset, mxrt::Dataset, std::shared_ptr<mxrt::SyntheticDataset>>(
      m, "SyntheticDataset")
      .def(pybind11::init<int, int, int, uint64_t>(), pybind11::arg("seq_len"), pybind11::arg("vocab"),
           pybind11::arg("doc_len"), pybind11::arg("seed"));
  pybind11::class_<mxrt::TokenSeqDataset, mxrt::Dataset, std::shared_ptr<mxrt::TokenSeqDataset>>(
      m, "TokenSeqDataset")
      .def(pybind11::init<const std::vector<std::string>&, const std::vector<std::string>&, int, uint64_t, bool,
                          const std::vector<std::string>&>(),
           pybind11::arg("token_files"), pybind11::arg("doc_files"), pybind11::arg("seq_len"),
           pybind11::arg("seed"), pybind11::arg("shuffle") = true,
           pybind11::arg("mask_files") = std::vector<std::string>())
      .def("total_tokens", &mxrt::TokenSeqDataset::total_tokens);
  pybind11::class_<mxrt::MixtureDataset, mxrt::Dataset, std::shared_ptr<mxrt::MixtureDataset>>(m, "MixtureDataset")
      .def(pybind11::init([](std::vector<std::shared_ptr<mxrt::Dataset>> comps, std::vector<uint64_t> starts,
                             std::vector<std::vector<double>> weights, uint64_t block, uint64_t seed, int stop) {
             return std::make_shared<mxrt::MixtureDataset>(std::move(comps), std::move(starts), std::move(weights),
                                                           block, seed, static_cast<mxrt::StopStrategy>(stop));
           }),
           pybind11::arg("components"), pybind11::arg("stage_starts"), pybind11::arg("stage_weights"),
           pybind11::arg("block_size"), pybind11::arg("seed"), pybind11::arg("stop") = 0)
      .def("resolve", [](const mxrt::MixtureDataset& d, uint64_t idx) {
        int c;
        uint64_t local;
        d.resolve(idx, c, local);
        return std::make_pair(c, local);
      });
  m.def("permutation", [](uint64_t n, uint64_t key, uint64_t i) { return mxrt::Permutation(n, key)(i); });

  pybind11::class_<PyPrefetcher, std::shared_ptr<PyPrefetcher>>(m, "Prefetcher")
      .def(pybind11::init([](std::shared_ptr<mxrt::Dataset> ds, int local_batch, int global_batch, int rank,
                             uint64_t start_step, std::vector<at::Tensor> tok, std::vector<at::Tensor> seg,
                             std::vector<at::Tensor> lw, int threads) {
             auto out = std::make_shared<PyPrefetcher>();
             std::vector<int32_t*> t, s;
             std::vector<float*> w;
             for (size_t i = 0; i < tok.size(); ++i) {
               check_batch(*ds, tok[i], seg.at(i), lw.at(i));
               TORCH_CHECK(tok[i].size(0) == local_batch, "slot buffers must hold the local batch");
               t.push_back(tok[i].data_ptr<int32_t>());
               s.push_back(seg[i].data_ptr<int32_t>());
               w.push_back(lw[i].data_ptr<float>());
               out->keep.push_back(tok[i]);
               out->keep.push_back(seg[i]);
               out->keep.push_back(lw[i]);
             }
             out->pf = std::make_unique<mxrt::Prefetcher>(ds, local_batch, global_batch, rank, start_step, t, s, w,
                                                          threads);
             return out;
           }))
      .def("next",
           [](PyPrefetcher& p, double timeout_s) {
             if (!p.pf) throw std::runtime_error("prefetcher closed");
             uint64_t step = 0;
             int slot;
             {
               pybind11::gil_scoped_release nogil;
               slot = p.pf->next(timeout_s, step);
             }
             return std::make_pair(slot, step);
           },
           pybind11::arg("timeout_s") = 600.0)
      .def("close",
           [](PyPrefetcher& p) {
             pybind11::gil_scoped_release nogil;
             p.pf.reset();
           })
      .def("release", [](PyPrefetcher& p, int slot) {
        if (p.pf) p.pf->release(slot);
      });
}
