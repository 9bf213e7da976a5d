// gawee-cuda-runner: the reference runner's file contract on a B200.
//
//   gawee-cuda-runner <model.mlir> <inputs_dir> <outputs_dir>
//                     [--entry forward] [--device 0] [--iters N]
//
// Reads argN.npy for every `forward` argument, runs the graph with
// libgawee_cuda, and writes outputN.npy — the same files the reference's
// generated runner reads and writes (back/gawee_aot.cpp:226-289), so
// `gawee-eval compare` / `benchmark` (back/gawee_eval.cpp) work unchanged.
// With --iters N > 1 it also prints the mean in-process time of N forwards.
#include <chrono>
#include <cstring>
#include <filesystem>
#include <iostream>
#include <string>
#include <vector>

#include "gawee_cuda.h"
#include "../host/npy.h"

namespace fs = std::filesystem;

static int fail(gawee_ctx* ctx, gawee_status st, const char* what) {
  char buf[2048];
  gawee_last_error(ctx, buf, sizeof(buf));
  std::cerr << "gawee-cuda-runner: " << what << " failed (status " << st << "): " << buf << "\n";
  return 1;
}

int main(int argc, char** argv) {
  if (argc < 4) {
    std::cerr << "Usage: " << argv[0] << " <model.mlir> <inputs_dir> <outputs_dir> [--entry forward] [--device 0] [--iters N]\n";
    return 1;
  }
  std::string entry = "forward";
  int device = 0, iters = 1;
  for (int i = 4; i < argc; ++i) {
    if (!std::strcmp(argv[i], "--entry") && i + 1 < argc) entry = argv[++i];
    else if (!std::strcmp(argv[i], "--device") && i + 1 < argc) device = std::atoi(argv[++i]);
    else if (!std::strcmp(argv[i], "--iters") && i + 1 < argc) iters = std::max(1, std::atoi(argv[++i]));
  }
  gawee_ctx* ctx = nullptr;
  gawee_status st = gawee_create_from_file(argv[1], entry.c_str(), device, &ctx);
  if (st) return fail(nullptr, st, "planning");
  try {
    int nargs = gawee_num_args(ctx);
    std::vector<gawee::NpyArray> args;
    for (int a = 0; a < nargs; ++a) {
      int dt, rank;
      int64_t shape[8];
      gawee_arg_info(ctx, a, &dt, &rank, shape);
      auto arr = gawee::npy_load((fs::path(argv[2]) / ("arg" + std::to_string(a) + ".npy")).string());
      if ((int)arr.dtype != dt || (int)arr.shape.size() != rank ||
          !std::equal(arr.shape.begin(), arr.shape.end(), shape))
        throw std::runtime_error("arg" + std::to_string(a) + ".npy does not match the forward signature");
      st = gawee_set_arg(ctx, a, arr.data.data(), arr.data.size(), nullptr);
      if (st) return fail(ctx, st, "staging");
      args.push_back(std::move(arr));
    }
    st = gawee_forward(ctx, nullptr);
    if (!st) st = gawee_synchronize(ctx, nullptr);
    if (st) return fail(ctx, st, "forward");
    if (iters > 1) {
      auto t0 = std::chrono::steady_clock::now();
      for (int i = 0; i < iters; ++i) {
        for (int a = 0; a < nargs; ++a) gawee_set_arg(ctx, a, args[a].data.data(), args[a].data.size(), nullptr);
        st = gawee_forward(ctx, nullptr);
        if (st) return fail(ctx, st, "forward");
      }
      st = gawee_synchronize(ctx, nullptr);
      if (st) return fail(ctx, st, "forward");
      auto t1 = std::chrono::steady_clock::now();
      std::cerr << "[gawee-cuda] mean_ms=" << std::chrono::duration<double, std::milli>(t1 - t0).count() / iters << "\n";
    }
    fs::create_directories(argv[3]);
    for (int r = 0; r < gawee_num_outputs(ctx); ++r) {
      int dt, rank;
      int64_t shape[8];
      gawee_output_info(ctx, r, &dt, &rank, shape);
      std::vector<int64_t> sh(shape, shape + rank);
      int64_t n = 1;
      for (auto d : sh) n *= d;
      std::vector<uint8_t> host((size_t)n * gawee::dtype_size((gawee::DType)dt));
      st = gawee_get_output(ctx, r, host.data(), host.size(), nullptr);
      if (!st) st = gawee_synchronize(ctx, nullptr);
      if (st) return fail(ctx, st, "reading outputs");
      gawee::npy_save((fs::path(argv[3]) / ("output" + std::to_string(r) + ".npy")).string(), (gawee::DType)dt, sh,
                      host.data());
    }
  } catch (const std::exception& e) {
    std::cerr << "gawee-cuda-runner: " << e.what() << "\n";
    gawee_destroy(ctx);
    return 1;
  }
  gawee_destroy(ctx);
  return 0;
}
