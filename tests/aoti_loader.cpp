// Runs an AOTInductor package of a batch tensor product from C++ (test helper for
// tests/test_export_gpu.py::test_aoti_cpp_loader).
//
// Usage: aoti_loader <package.pt2> <dir> <batch> <L1_dim> <L2_dim> <weight_numel> <L3_dim>
// Reads <dir>/{x,y,w}.bin (float32, row-major), runs the package on the GPU and writes
// <dir>/z.bin.  The program is linked against libtorch_oeqb200.so (with --no-as-needed), whose
// static initialisers register the libtorch_tp_jit operators the package calls.
#include <torch/torch.h>
#include <torch/csrc/inductor/aoti_package/model_package_loader.h>

#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <string>
#include <vector>

namespace {

at::Tensor read_rows(const std::string& path, int64_t rows, int64_t cols) {
  std::vector<float> buf(static_cast<size_t>(rows * cols));
  std::ifstream f(path, std::ios::binary);
  if (!f.read(reinterpret_cast<char*>(buf.data()), static_cast<std::streamsize>(buf.size() * 4))) {
    std::fprintf(stderr, "cannot read %s\n", path.c_str());
    std::exit(2);
  }
  return torch::from_blob(buf.data(), {rows, cols}, torch::kFloat32).clone().to(torch::kCUDA);
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 8) {
    std::fprintf(stderr, "usage: %s package dir batch L1 L2 W L3\n", argv[0]);
    return 2;
  }
  const std::string pkg = argv[1], dir = argv[2];
  const int64_t B = std::atoll(argv[3]), d1 = std::atoll(argv[4]), d2 = std::atoll(argv[5]),
                wn = std::atoll(argv[6]), d3 = std::atoll(argv[7]);
  torch::NoGradGuard no_grad;
  torch::inductor::AOTIModelPackageLoader loader(pkg);
  std::vector<at::Tensor> inputs = {read_rows(dir + "/x.bin", B, d1),
                                    read_rows(dir + "/y.bin", B, d2),
                                    read_rows(dir + "/w.bin", B, wn)};
  std::vector<at::Tensor> out = loader.run(inputs);
  if (out.size() != 1 || out[0].size(0) != B || out[0].size(1) != d3) {
    std::fprintf(stderr, "unexpected output\n");
    return 3;
  }
  at::Tensor z = out[0].to(torch::kCPU).contiguous();
  std::ofstream f(dir + "/z.bin", std::ios::binary);
  f.write(reinterpret_cast<const char*>(z.data_ptr<float>()),
          static_cast<std::streamsize>(z.numel() * 4));
  std::printf("ok %lld x %lld\n", static_cast<long long>(z.size(0)),
              static_cast<long long>(z.size(1)));
  return 0;
}
