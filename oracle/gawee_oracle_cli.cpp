// gawee-oracle: run a gawee-dialect graph on the CPU oracle with the reference
// runner's file contract (back/gawee_aot.cpp:226-289): read argN.npy from an
// inputs directory, write outputN.npy to an outputs directory.
// TEST INFRASTRUCTURE ONLY.
//
//   gawee-oracle <model.mlir> <inputs_dir> <outputs_dir> [--entry forward] [--threads N]
#include <chrono>
#include <cstring>
#include <filesystem>
#include <iostream>

#include "../gawee_b200/csrc/host/ir.h"
#include "../gawee_b200/csrc/host/npy.h"

extern "C" {
void* gawee_oracle_load(const char* mlir_text, const char* entry, char* err, int errlen);
int gawee_oracle_run(void* h, const void* const* args, void* const* outs, int threads, char* err, int errlen);
void gawee_oracle_free(void* h);
}

int main(int argc, char** argv) {
  namespace fs = std::filesystem;
  if (argc < 4) {
    std::cerr << "Usage: " << argv[0] << " <model.mlir> <inputs_dir> <outputs_dir> [--entry forward] [--threads N]\n";
    return 1;
  }
  std::string entry = "forward";
  int threads = 0;
  for (int i = 4; i < argc; ++i) {
    if (!std::strcmp(argv[i], "--entry") && i + 1 < argc) entry = argv[++i];
    else if (!std::strcmp(argv[i], "--threads") && i + 1 < argc) threads = std::atoi(argv[++i]);
  }
  try {
    std::string text = gawee::read_text_file(argv[1]);
    gawee::Graph g = gawee::parse_mlir(text, entry);
    std::vector<gawee::NpyArray> ins;
    std::vector<const void*> ptrs;
    for (size_t a = 0; a < g.args.size(); ++a) {
      ins.push_back(gawee::npy_load((fs::path(argv[2]) / ("arg" + std::to_string(a) + ".npy")).string()));
      const auto& t = g.values[g.args[a]].type;
      if (ins.back().dtype != t.dtype || ins.back().shape != t.shape)
        throw std::runtime_error("arg" + std::to_string(a) + ".npy does not match " + t.str());
    }
    for (auto& a : ins) ptrs.push_back(a.data.data());
    std::vector<std::vector<uint8_t>> outs;
    std::vector<void*> optr;
    for (int r : g.results) {
      outs.emplace_back((size_t)g.values[r].type.numel() * gawee::dtype_size(g.values[r].type.dtype));
      optr.push_back(outs.back().data());
    }
    char err[1024] = {0};
    void* h = gawee_oracle_load(text.c_str(), entry.c_str(), err, sizeof(err));
    if (!h) throw std::runtime_error(err);
    auto t0 = std::chrono::steady_clock::now();
    int rc = gawee_oracle_run(h, ptrs.data(), optr.data(), threads, err, sizeof(err));
    auto t1 = std::chrono::steady_clock::now();
    gawee_oracle_free(h);
    if (rc) throw std::runtime_error(err);
    fs::create_directories(argv[3]);
    for (size_t r = 0; r < g.results.size(); ++r) {
      const auto& t = g.values[g.results[r]].type;
      gawee::npy_save((fs::path(argv[3]) / ("output" + std::to_string(r) + ".npy")).string(), t.dtype, t.shape,
                      outs[r].data());
    }
    std::cerr << "[gawee-oracle] compute_ms=" << std::chrono::duration<double, std::milli>(t1 - t0).count() << "\n";
    return 0;
  } catch (std::exception& e) {
    std::cerr << "gawee-oracle error: " << e.what() << "\n";
    return 1;
  }
}
