// Drives neon_cuda::proj_all_positions[_multi] (the C++ drop-in header) the
// way transformer_forward() calls fwd::proj_all_positions[_multi]: tensor
// handles with loader::TensorInfo's public fields, host X and Y, a pool
// argument. Reads raw inputs from files, writes outputs to files.
//
//   shim_driver single <type> <rows> <cols> <seq> W.bin X.bin Y.out
//   shim_driver multi  <cols> <seq> X.bin Y.out <type> <rows> W.bin [<type> <rows> W.bin ...]
//   shim_driver badshape       (expects the reference's error message)
//   shim_driver roles <name>...  (GGUF tensor name -> "role layer", or "none")
//   shim_driver decode <dir> <n_new> [quantize_to]
//       builds neon_cuda::Decoder from <dir>/config.txt (engine::Config fields),
//       <dir>/manifest.txt ("name type ne0 ne1 file" per tensor) and
//       <dir>/prompt.bin (int32); writes tokens.bin (greedy generation) and
//       logits.bin (forward of the prompt after a rewind to 0)
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iostream>
#include <iterator>
#include <string>
#include <vector>

#include "neon_proj_cuda.hpp"

namespace loader {
enum class GGMLType : uint32_t { F32 = 0, F16 = 1, Q4_0 = 2, Q8_0 = 8 };
struct TensorInfo {  // public fields of loader::TensorInfo (rawllm_loader.hpp:34-41)
    std::string name;
    std::vector<uint64_t> shape;
    GGMLType type;
    uint64_t file_offset = 0;
    size_t nbytes = 0;
    const uint8_t* data_ptr = nullptr;
};
}  // namespace loader

namespace fwd {
struct ProjTarget {  // fwd::ProjTarget (rawllm_forward.hpp:626-630)
    const loader::TensorInfo* W;
    float* Y;
    size_t y_stride;
};
}  // namespace fwd

namespace engine {
struct Config {  // the fields of engine::Config the decoder reads (rawllm_common.hpp:113-145)
    uint32_t n_vocab = 0, n_embd = 0, n_layer = 0, n_head = 0, n_kv_head = 0, head_dim = 0, n_ff = 0;
    uint32_t ctx_len = 4096, kv_window = 0;
    float rope_base = 10000.f, rope_scale = 1.f;
    uint32_t rope_dim_count = 0;
    float norm_eps = 1e-5f;
    bool use_swiglu = true;
};
}  // namespace engine

struct Loader {  // a loader's public tensor list (GGUFLoader::tensors)
    std::vector<loader::TensorInfo> tensors;
};

struct DummyPool {
    int size() const { return 1; }
};

static std::vector<uint8_t> read_file(const char* p) {
    std::ifstream f(p, std::ios::binary);
    return std::vector<uint8_t>(std::istreambuf_iterator<char>(f), {});
}

static void write_file(const char* p, const float* y, size_t n) {
    std::ofstream f(p, std::ios::binary);
    f.write(reinterpret_cast<const char*>(y), n * sizeof(float));
}

int main(int argc, char** argv) {
    if (argc < 2) return 2;
    DummyPool pool;
    try {
        std::string mode = argv[1];
        if (mode == "badshape") {
            std::vector<uint8_t> bytes(64);
            loader::TensorInfo t{"blk.3.attn_k.weight", {100, 2}, loader::GGMLType::Q4_0, 0, 64, bytes.data()};
            std::vector<float> X(100), Y(2);
            try {
                neon_cuda::proj_all_positions(t, X.data(), 100, Y.data(), 2, 1, pool);
            } catch (const std::runtime_error& e) {
                std::cout << e.what() << "\n";
                return 0;
            }
            return 1;
        }
        if (mode == "roles") {
            for (int i = 2; i < argc; ++i) {
                int role = 0, layer = 0;
                if (neon_cuda::tensor_role(argv[i], &role, &layer)) std::cout << role << " " << layer << "\n";
                else std::cout << "none\n";
            }
            return 0;
        }
        if (mode == "decode" && (argc == 4 || argc == 5)) {
            const std::string dir = argv[2];
            const size_t n_new = std::strtoull(argv[3], nullptr, 10);
            const int quantize_to = argc == 5 ? std::atoi(argv[4]) : -1;
            engine::Config cfg;
            {
                std::ifstream f(dir + "/config.txt");
                int swiglu = 1;
                f >> cfg.n_vocab >> cfg.n_embd >> cfg.n_layer >> cfg.n_head >> cfg.n_kv_head >> cfg.head_dim >> cfg.n_ff >>
                    cfg.ctx_len >> cfg.kv_window >> cfg.rope_base >> cfg.rope_scale >> cfg.rope_dim_count >> cfg.norm_eps >>
                    swiglu;
                cfg.use_swiglu = swiglu != 0;
            }
            Loader g;
            std::vector<std::vector<uint8_t>> blobs;
            {
                std::ifstream f(dir + "/manifest.txt");
                std::string name, file;
                int type;
                uint64_t ne0, ne1;
                while (f >> name >> type >> ne0 >> ne1 >> file) {
                    blobs.push_back(read_file((dir + "/" + file).c_str()));
                    loader::TensorInfo t{name, ne1 ? std::vector<uint64_t>{ne0, ne1} : std::vector<uint64_t>{ne0},
                                         static_cast<loader::GGMLType>(type), 0, blobs.back().size(), nullptr};
                    g.tensors.push_back(t);
                }
                for (size_t i = 0; i < g.tensors.size(); ++i) g.tensors[i].data_ptr = blobs[i].data();
            }
            auto pb = read_file((dir + "/prompt.bin").c_str());
            std::vector<int32_t> prompt(pb.size() / 4);
            std::memcpy(prompt.data(), pb.data(), pb.size());
            neon_cuda::check(neon_cuda_init(0));
            neon_cuda::Decoder d(cfg, g, nullptr, quantize_to);
            auto toks = d.generate(prompt, n_new, -1);
            {
                std::ofstream f(dir + "/tokens.bin", std::ios::binary);
                f.write(reinterpret_cast<const char*>(toks.data()), toks.size() * 4);
            }
            if (d.length() != prompt.size() + toks.size()) return 5;
            d.set_length(0);
            auto logits = d.forward(prompt, cfg.n_vocab);
            write_file((dir + "/logits.bin").c_str(), logits.data(), logits.size());
            return 0;
        }
        if (mode == "single" && argc == 9) {
            int type = std::atoi(argv[2]);
            size_t rows = std::strtoull(argv[3], nullptr, 10), cols = std::strtoull(argv[4], nullptr, 10),
                   seq = std::strtoull(argv[5], nullptr, 10);
            auto W = read_file(argv[6]);
            auto Xb = read_file(argv[7]);
            loader::TensorInfo t{"w", {cols, rows}, static_cast<loader::GGMLType>(type), 0, W.size(), W.data()};
            std::vector<float> Y(seq * rows);
            neon_cuda::proj_all_positions(t, reinterpret_cast<const float*>(Xb.data()), cols, Y.data(), rows, seq,
                                          pool);
            // a second call reuses the uploaded tensor
            neon_cuda::proj_all_positions(t, reinterpret_cast<const float*>(Xb.data()), cols, Y.data(), rows, seq,
                                          pool);
            if (neon_cuda::tensors().size() != 1) return 3;
            write_file(argv[8], Y.data(), Y.size());
            return 0;
        }
        if (mode == "multi" && argc >= 9 && (argc - 6) % 3 == 0) {
            size_t cols = std::strtoull(argv[2], nullptr, 10), seq = std::strtoull(argv[3], nullptr, 10);
            auto Xb = read_file(argv[4]);
            size_t n = (argc - 6) / 3;
            std::vector<std::vector<uint8_t>> Ws(n);
            std::vector<loader::TensorInfo> ts(n);
            std::vector<std::vector<float>> Ys(n);
            std::vector<fwd::ProjTarget> targets;
            for (size_t i = 0; i < n; ++i) {
                int type = std::atoi(argv[6 + 3 * i]);
                size_t rows = std::strtoull(argv[7 + 3 * i], nullptr, 10);
                Ws[i] = read_file(argv[8 + 3 * i]);
                ts[i] = loader::TensorInfo{"t" + std::to_string(i), {cols, rows}, static_cast<loader::GGMLType>(type),
                                           0, Ws[i].size(), Ws[i].data()};
                Ys[i].assign(seq * rows, 0.f);
            }
            for (size_t i = 0; i < n; ++i) targets.push_back({&ts[i], Ys[i].data(), (size_t)ts[i].shape[1]});
            neon_cuda::proj_all_positions_multi(targets, reinterpret_cast<const float*>(Xb.data()), cols, seq, pool);
            std::vector<float> all;
            for (auto& y : Ys) all.insert(all.end(), y.begin(), y.end());
            write_file(argv[5], all.data(), all.size());
            return 0;
        }
    } catch (const std::exception& e) {
        std::cerr << "error: " << e.what() << "\n";
        return 4;
    }
    return 2;
}
