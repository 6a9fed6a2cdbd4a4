// ref_harness.cu -- dumps logits computed by the REFERENCE's own CUDA model
// (BoaPredictorGPU from portability_solved_cpp/boa_gpu.hpp, compiled from the
// reference sources where they lie by oracle/build_ref.sh).  Test
// infrastructure: it produces the golden logits that pin the CPU oracle.
//
// usage: ref_logits <weights.bin> <backbone> <d_model> <n_layers> <tokens.u8> <B> <T> <mode> <out.f32>
//   tokens.u8 holds B*T bytes (row-major [B][T]); mode = chunk | step.
//   chunk: BoaPredictorGPU::forward_chunk (boa_gpu.hpp:1081) over T tokens.
//   step : BoaPredictorGPU::step_batch (boa_gpu.hpp:1034) T times, head bias on.
//   out.f32 receives [B][T][256] float32 logits.
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>
#include "boa_gpu.hpp"

int main(int argc, char** argv) {
  if (argc != 10) { fprintf(stderr, "usage: see header\n"); return 2; }
  std::string wpath = argv[1];
  MambaConfig cfg;
  cfg.d_model = atoi(argv[3]);
  cfg.n_layers = atoi(argv[4]);
  cfg.backbone = backbone_from_string(argv[2]);
  cfg.update();
  cfg.use_rmsnorm = false;  // boa.cpp:920
  int B = atoi(argv[6]), T = atoi(argv[7]);
  std::string mode = argv[8];
  std::vector<uint8_t> tok((size_t)B * T);
  FILE* f = fopen(argv[5], "rb");
  if (!f || fread(tok.data(), 1, tok.size(), f) != tok.size()) { fprintf(stderr, "tokens\n"); return 3; }
  fclose(f);
  BoaPredictorGPU model(cfg, 256, cfg.n_layers, B);
  model.load_weights(wpath);
  std::vector<float> out((size_t)B * T * 256);
  float* d_logits = nullptr;
  int* d_tok = nullptr;
  if (mode == "chunk") {
    model.allocate_chunk(T);
    std::vector<int> ti(tok.begin(), tok.end());
    checkCudaErrors(cudaMalloc(&d_tok, ti.size() * sizeof(int)));
    checkCudaErrors(cudaMalloc(&d_logits, out.size() * sizeof(float)));
    checkCudaErrors(cudaMemcpy(d_tok, ti.data(), ti.size() * sizeof(int), cudaMemcpyHostToDevice));
    model.reset_cache();
    model.forward_chunk(d_tok, d_logits, T);
    checkCudaErrors(cudaDeviceSynchronize());
    checkCudaErrors(cudaMemcpy(out.data(), d_logits, out.size() * sizeof(float), cudaMemcpyDeviceToHost));
  } else {
    checkCudaErrors(cudaMalloc(&d_tok, B * sizeof(int)));
    checkCudaErrors(cudaMalloc(&d_logits, (size_t)B * 256 * sizeof(float)));
    std::vector<int> step(B);
    std::vector<float> lg((size_t)B * 256);
    model.reset_cache();
    for (int t = 0; t < T; ++t) {
      for (int b = 0; b < B; ++b) step[b] = tok[(size_t)b * T + t];
      checkCudaErrors(cudaMemcpy(d_tok, step.data(), B * sizeof(int), cudaMemcpyHostToDevice));
      model.step_batch(d_tok, d_logits, true);
      checkCudaErrors(cudaDeviceSynchronize());
      checkCudaErrors(cudaMemcpy(lg.data(), d_logits, lg.size() * sizeof(float), cudaMemcpyDeviceToHost));
      for (int b = 0; b < B; ++b)
        std::copy(lg.begin() + (size_t)b * 256, lg.begin() + (size_t)(b + 1) * 256,
                  out.begin() + ((size_t)b * T + t) * 256);
    }
  }
  FILE* o = fopen(argv[9], "wb");
  fwrite(out.data(), sizeof(float), out.size(), o);
  fclose(o);
  return 0;
}
