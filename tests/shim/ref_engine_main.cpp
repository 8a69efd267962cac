// ref_engine_main.cpp - runs the reference's own decode engine with its matrix-product path on
// the GPU. The reference's src/model.cpp, qfile.cpp, kernels.cpp, json.cpp, mapped_file.cpp,
// model_config.cpp, safetensors.cpp and threadpool.cpp are compiled unchanged, except that
// their ef/quant.h and ef/qkernels.h resolve to include/shim/ef/*.h (include/efg_ref_shim.hpp
// over libefg.so); src/quant.cpp and src/qkernels.cpp are not built. Test infrastructure for
// tests/test_ref_engine_gpu.py (recipe: tests/shim/Makefile).
//
//   ref_engine <model.efq> <prompt ids> <forced ids> <out.f32> [dequantized]
//
// Ids are comma-separated. Teacher-forced like the reference's bench_decode: the prompt from
// position 0, then each forced id in turn. Writes the logits after the last prompt token and
// after each forced id but the last ([len(forced)][vocab] floats, native byte order). With
// "dequantized" the engine runs on Model::dequantized_copy, whose weights are F32 views (the
// plain-type matvec path). The packed views are registered with efg_host_register_weights
// first, as an integration does once at load, so each call moves only x and y.
#include <cstdio>
#include <cstdlib>
#include <sstream>
#include <string>
#include <vector>

#include "ef/model.h"
#include "efg.h"

namespace {

std::vector<std::int32_t> parse_ids(const std::string& s) {
  std::vector<std::int32_t> v;
  std::stringstream ss(s);
  std::string item;
  while (std::getline(ss, item, ','))
    if (!item.empty()) v.push_back(static_cast<std::int32_t>(std::stol(item)));
  return v;
}

void register_view(const ef::WeightView& w) {
  if (w.data && w.rows && w.cols) efg_host_register_weights(w.data, static_cast<size_t>(w.bytes()));
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 5) {
    std::fprintf(stderr, "usage: %s <model.efq> <prompt ids> <forced ids> <out.f32> [dequantized]\n", argv[0]);
    return 2;
  }
  try {
    const std::vector<std::int32_t> prompt = parse_ids(argv[2]), forced = parse_ids(argv[3]);
    const bool deq = argc > 5 && std::string(argv[5]) == "dequantized";
    const ef::Model packed = ef::Model::load_efq(argv[1]);
    const ef::Model model = deq ? ef::Model::dequantized_copy(packed) : ef::Model();
    const ef::Model& m = deq ? model : packed;
    register_view(m.lm_head());
    for (std::size_t l = 0; l < m.n_layers(); ++l) {
      const ef::LayerWeights& w = m.layer(l);
      for (const ef::WeightView* v : {&w.wq, &w.wk, &w.wv, &w.wo, &w.w_gate, &w.w_up, &w.w_down}) register_view(*v);
    }
    ef::Transformer t(m, prompt.size() + forced.size());
    const std::size_t vocab = static_cast<std::size_t>(m.config().vocab_size);
    std::vector<float> out;
    std::size_t pos = 0;
    const float* lg = nullptr;
    for (std::size_t i = 0; i < prompt.size(); ++i) lg = t.forward(prompt[i], pos++, i + 1 == prompt.size());
    out.insert(out.end(), lg, lg + vocab);
    for (std::size_t i = 0; i + 1 < forced.size(); ++i) {
      lg = t.forward(forced[i], pos++);
      out.insert(out.end(), lg, lg + vocab);
    }
    efg_host_release_weights();
    FILE* f = std::fopen(argv[4], "wb");
    if (!f || std::fwrite(out.data(), sizeof(float), out.size(), f) != out.size()) {
      std::fprintf(stderr, "cannot write %s\n", argv[4]);
      return 1;
    }
    std::fclose(f);
    std::printf("%s: %zu logit rows of %zu, %s\n", m.description().c_str(), out.size() / vocab, vocab,
                deq ? "dequantized F32 views" : "packed views");
  } catch (const ef::Error& e) {
    std::fprintf(stderr, "ef::Error: %s\n", e.what());
    return 1;
  }
  return 0;
}
