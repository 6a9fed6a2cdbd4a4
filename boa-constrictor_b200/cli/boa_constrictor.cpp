// boa_constrictor -- command-line front end with the reference CLI's surface
// (portability_solved_cpp/boa.cpp:819-942):
//
//   boa_constrictor <compress|decompress> <model.bin> <input> <output>
//                   [d_model] [n_layers] [--backbone mamba|lstm|gru|mingru]
//                   [--gpu-batch B] [--max-chunks C] [--chunk-size S] [--tile T]
//                   [--temperature T] [--show-timings] [--no-graph] [--gpus N]
//
// Defaults follow the reference: d_model 256, n_layers 1, chunk 4096.  The
// extra --gpus N shards the chunks over N GPUs of this node (contiguous chunk
// ranges, one host thread and one library handle per GPU); the container is
// the same BOA2 file either way.  --warm-start (one GPU only) runs W lanes
// that carry the model state from each chunk into the next one of the same
// lane (boa.cpp:313-319); the container records W for decompress.
#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iostream>
#include <string>
#include <thread>
#include <vector>

#include "boa_b200.h"

namespace {

struct Opts {
  std::string mode, model, in, out, backbone = "mamba";
  int d_model = 256, n_layers = 1, gpu_batch = 0, max_chunks = -1, tile = 0, gpus = 1;
  size_t chunk = 4096;
  float temperature = 1.0f;
  bool timings = false, warm = false;
};

bool read_file(const std::string& p, std::vector<uint8_t>& v) {
  std::ifstream f(p, std::ios::binary);
  if (!f) return false;
  v.assign(std::istreambuf_iterator<char>(f), std::istreambuf_iterator<char>());
  return true;
}

int backbone_code(const std::string& s) {
  if (s == "mamba" || s == "mambav1") return BOA_BACKBONE_MAMBA;
  if (s == "lstm") return BOA_BACKBONE_LSTM;
  if (s == "gru") return BOA_BACKBONE_GRU;
  if (s == "mingru") return BOA_BACKBONE_MINGRU;
  return -1;
}

struct Shard {
  uint32_t c0, n;
};
std::vector<Shard> shards(uint32_t n_chunks, int gpus) {
  std::vector<Shard> s;
  for (int g = 0; g < gpus; ++g) {
    uint32_t a = (uint32_t)((uint64_t)n_chunks * g / gpus), b = (uint32_t)((uint64_t)n_chunks * (g + 1) / gpus);
    if (b > a) s.push_back({a, b - a});
  }
  return s;
}

int open_model(const Opts& o, int dev, boa_model** h) {
  int rc = boa_model_load(o.model.c_str(), backbone_code(o.backbone), o.d_model, o.n_layers, dev, h);
  if (rc) { std::cerr << "Error: " << boa_last_error(nullptr) << "\n"; return rc; }
  if (o.temperature != 1.0f) boa_set_temperature(*h, o.temperature);
  boa_set_batch(*h, o.gpu_batch, o.tile);
  return 0;
}

int do_compress(const Opts& o) {
  std::vector<uint8_t> data;
  if (!read_file(o.in, data)) { std::cerr << "Error: cannot read " << o.in << "\n"; return 1; }
  const size_t total = data.size();
  if (total == 0) { std::cerr << "Error: empty input\n"; return 1; }
  uint32_t n_chunks = (uint32_t)((total + o.chunk - 1) / o.chunk);
  if (o.max_chunks > 0 && (uint32_t)o.max_chunks < n_chunks) n_chunks = (uint32_t)o.max_chunks;
  const size_t processed = std::min(total, (size_t)n_chunks * o.chunk);  // boa.cpp:299
  const uint32_t last = (uint32_t)(n_chunks > 1 ? processed - (size_t)(n_chunks - 1) * o.chunk : processed);
  std::cout << "Compressing " << processed << " bytes in " << n_chunks << " chunks on " << o.gpus << " GPU(s)..."
            << std::endl;
  uint32_t warm_w = 0;
  if (o.warm) {
    if (o.gpus != 1) { std::cerr << "Error: --warm-start needs --gpus 1\n"; return 1; }
    warm_w = (uint32_t)std::min<uint64_t>(o.gpu_batch > 0 ? o.gpu_batch : 64, n_chunks);  // boa.cpp:310-311
    std::cout << "Warm start: " << warm_w << " lanes" << std::endl;
  }
  std::vector<uint8_t> first(n_chunks);
  std::vector<uint32_t> sizes(n_chunks);
  const auto sh = shards(n_chunks, o.gpus);
  std::vector<std::vector<uint32_t>> pay(sh.size());
  std::vector<int> rcs(sh.size(), 0);
  auto t0 = std::chrono::steady_clock::now();
  std::vector<std::thread> th;
  for (size_t g = 0; g < sh.size(); ++g)
    th.emplace_back([&, g]() {
      boa_model* h = nullptr;
      if ((rcs[g] = open_model(o, (int)g, &h))) return;
      if (warm_w) boa_set_warm_start(h, warm_w);
      const Shard s = sh[g];
      size_t cap = (size_t)s.n * boa_stream_capacity_words((uint32_t)o.chunk);
      pay[g].resize(cap);
      uint64_t used = 0;
      rcs[g] = boa_compress_chunks(h, data.data(), processed, (uint32_t)o.chunk, s.c0, s.n, first.data() + s.c0,
                                   pay[g].data(), cap, sizes.data() + s.c0, &used);
      if (rcs[g]) std::cerr << "Error (GPU " << g << "): " << boa_last_error(h) << "\n";
      pay[g].resize(used);
      boa_model_free(h);
    });
  for (auto& t : th) t.join();
  for (int rc : rcs)
    if (rc) return 1;
  const double secs = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  std::vector<uint8_t> payload;
  for (auto& p : pay) payload.insert(payload.end(), (uint8_t*)p.data(), (uint8_t*)(p.data() + p.size()));
  std::vector<uint64_t> sb(n_chunks);
  for (uint32_t i = 0; i < n_chunks; ++i) sb[i] = (uint64_t)sizes[i] * 4;
  size_t len = 0;
  const uint32_t flags = warm_w ? 1u : 0u;
  boa_boa2_build(processed, (uint32_t)o.chunk, n_chunks, last, flags, warm_w, first.data(), sb.data(), payload.data(),
                 nullptr, 0, &len);
  std::vector<uint8_t> blob(len);
  if (boa_boa2_build(processed, (uint32_t)o.chunk, n_chunks, last, flags, warm_w, first.data(), sb.data(),
                     payload.data(), blob.data(), blob.size(), &len)) {
    std::cerr << "Error: container build failed\n";
    return 1;
  }
  std::ofstream f(o.out, std::ios::binary);
  f.write((const char*)blob.data(), (std::streamsize)blob.size());
  if (!f) { std::cerr << "Error: cannot write " << o.out << "\n"; return 1; }
  std::cout << "Done. Time: " << secs << "s, Avg Throughput: " << processed / 1048576.0 / secs << " MB/s, "
            << 8.0 * blob.size() / processed << " bits/byte\n";
  return 0;
}

int do_decompress(const Opts& o) {
  std::vector<uint8_t> buf;
  if (!read_file(o.in, buf)) { std::cerr << "Error: cannot read " << o.in << "\n"; return 1; }
  boa2_info I;
  if (boa_boa2_parse(buf.data(), buf.size(), &I, nullptr, nullptr, nullptr)) {
    std::cerr << "Error: not a valid BOA2 container\n";
    return 1;
  }
  const uint32_t warm_w = (I.flags & 1u) ? I.interleave_batch : 0u;  // boa.cpp:608-610
  if (warm_w && o.gpus != 1) { std::cerr << "Error: warm-start containers decode on one GPU\n"; return 1; }
  if ((I.flags & 1u) && warm_w == 0) { std::cerr << "Error: warm-start container without its batch\n"; return 1; }
  const uint32_t n = I.n_chunks;
  std::vector<uint8_t> first(n);
  std::vector<uint64_t> off(n), len(n);
  if (boa_boa2_parse(buf.data(), buf.size(), &I, first.data(), off.data(), len.data())) {
    std::cerr << "Error: not a valid BOA2 container\n";
    return 1;
  }
  std::vector<uint32_t> sizes(n), lens(n, I.chunk_len);
  if (n) lens[n - 1] = I.last_chunk_len;
  std::vector<uint32_t> words;
  uint64_t stream_total = 0;
  for (uint32_t i = 0; i < n; ++i) {
    // every stream must lie inside the file and the payload must add up
    if (I.payload_offset > buf.size() || off[i] > buf.size() - I.payload_offset ||
        len[i] > buf.size() - I.payload_offset - off[i]) {
      std::cerr << "Error: stream " << i << " lies outside the container\n";
      return 1;
    }
    stream_total += len[i];
    if (len[i] % 4) { std::cerr << "Error: stream " << i << " is not a whole number of words\n"; return 1; }
    sizes[i] = (uint32_t)(len[i] / 4);
    const uint8_t* p = buf.data() + I.payload_offset + off[i];
    const size_t w0 = words.size();
    words.resize(w0 + sizes[i]);
    std::memcpy(words.data() + w0, p, len[i]);
  }
  if (stream_total > I.payload_bytes) {
    std::cerr << "Error: stream lengths exceed the payload\n";
    return 1;
  }
  std::vector<uint64_t> woff(n + 1, 0);
  for (uint32_t i = 0; i < n; ++i) woff[i + 1] = woff[i] + sizes[i];
  std::vector<uint8_t> out(I.total_size);
  std::cout << "Decompressing " << I.total_size << " bytes in " << n << " chunks on " << o.gpus << " GPU(s)..."
            << std::endl;
  const auto sh = shards(n, o.gpus);
  std::vector<int> rcs(sh.size(), 0);
  auto t0 = std::chrono::steady_clock::now();
  std::vector<std::thread> th;
  for (size_t g = 0; g < sh.size(); ++g)
    th.emplace_back([&, g]() {
      boa_model* h = nullptr;
      if ((rcs[g] = open_model(o, (int)g, &h))) return;
      if (warm_w) boa_set_warm_start(h, warm_w);
      const Shard s = sh[g];
      rcs[g] = boa_decompress_chunks(h, words.data() + woff[s.c0], sizes.data() + s.c0, first.data() + s.c0,
                                     lens.data() + s.c0, I.chunk_len, s.n, out.data() + (size_t)s.c0 * I.chunk_len);
      if (rcs[g]) std::cerr << "Error (GPU " << g << "): " << boa_last_error(h) << "\n";
      boa_model_free(h);
    });
  for (auto& t : th) t.join();
  for (int rc : rcs)
    if (rc) return 1;
  const double secs = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  std::ofstream f(o.out, std::ios::binary);
  f.write((const char*)out.data(), (std::streamsize)out.size());
  if (!f) { std::cerr << "Error: cannot write " << o.out << "\n"; return 1; }
  std::cout << "Done. Time: " << secs << "s, Avg Throughput: " << I.total_size / 1048576.0 / secs << " MB/s\n";
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 5) {
    std::cerr << "Usage: boa_constrictor <compress|decompress> <model> <input> <output> [d_model] [n_layers] "
                 "[--backbone mamba|lstm|gru|mingru] [--gpu-batch B] [--max-chunks C] [--chunk-size S] [--tile T] "
                 "[--temperature T] [--show-timings] [--no-graph] [--gpus N] [--warm-start]\n";
    return 1;
  }
  Opts o;
  std::vector<std::string> pos;
  for (int i = 1; i < argc; ++i) {
    std::string s = argv[i];
    auto next = [&](const char* name) -> const char* {
      if (i + 1 >= argc) { std::cerr << "Error: " << name << " needs a value\n"; std::exit(1); }
      return argv[++i];
    };
    try {
      if (s == "--gpu-batch") o.gpu_batch = std::stoi(next("--gpu-batch"));
      else if (s == "--max-chunks") o.max_chunks = std::stoi(next("--max-chunks"));
      else if (s == "--chunk-size") o.chunk = (size_t)std::stoull(next("--chunk-size"));
      else if (s == "--backbone") o.backbone = next("--backbone");
      else if (s == "--tile") o.tile = std::stoi(next("--tile"));
      else if (s == "--temperature") o.temperature = std::stof(next("--temperature"));
      else if (s == "--gpus") o.gpus = std::stoi(next("--gpus"));
      else if (s == "--show-timings") o.timings = true;
      else if (s == "--no-graph" || s == "--gpu") continue;
      else if (s == "--warm-start") o.warm = true;
      else if (s == "--measure-energy") { std::cerr << "Warning: --measure-energy is not supported; ignored.\n"; }
      else if (s.rfind("--", 0) == 0) std::cerr << "Warning: Unknown flag '" << s << "' ignored.\n";
      else pos.push_back(s);
    } catch (const std::exception&) {
      std::cerr << "Error: bad value for " << s << "\n";
      return 1;
    }
  }
  if (pos.size() < 4) { std::cerr << "Error: missing arguments\n"; return 1; }
  o.mode = pos[0]; o.model = pos[1]; o.in = pos[2]; o.out = pos[3];
  try {
    if (pos.size() > 4) o.d_model = std::stoi(pos[4]);
    if (pos.size() > 5) o.n_layers = std::stoi(pos[5]);
  } catch (const std::exception&) {
    std::cerr << "Error: bad d_model / n_layers\n";
    return 1;
  }
  if (backbone_code(o.backbone) < 0) { std::cerr << "Error: unsupported backbone " << o.backbone << "\n"; return 1; }
  if (o.chunk == 0 || o.chunk > (1u << 30)) { std::cerr << "Error: bad chunk size\n"; return 1; }
  if (o.gpus < 1) o.gpus = 1;
  if (o.temperature <= 0.f) { std::cerr << "Error: temperature must be > 0\n"; return 1; }
  if (o.mode == "compress") return do_compress(o);
  if (o.mode == "decompress") return do_decompress(o);
  std::cerr << "Unknown mode: " << o.mode << "\n";
  return 1;
}
