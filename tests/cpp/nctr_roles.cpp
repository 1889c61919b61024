// Compiles the package's C++ adapter (host/neon_proj_cuda.hpp) together with
// the reference's own loader::NCTRLoader (rawllm_nctr_loader.hpp, from the
// reference tree) and maps every tensor of a .nctr file to the decoder role
// neon_cuda::Decoder would give it. No device is touched.
//   usage: nctr_roles <file.nctr>   -> one line per tensor: name role layer ne0 ne1 type nbytes
#include <cstdio>

#include "neon_proj_cuda.hpp"
#include "rawllm_nctr_loader.hpp"

int main(int argc, char** argv) {
    if (argc < 2) return 2;
    try {
        loader::NCTRLoader model;
        model.open(argv[1]);
        engine::Config cfg;
        model.validate_config(cfg);
        const neon_model_config_t c = neon_cuda::model_config(cfg);
        std::printf("config %u %u %u %u %u %u %u %u %u\n", c.n_vocab, c.n_embd, c.n_layer, c.n_head, c.n_kv_head,
                    c.head_dim, c.n_ff, c.ctx_len, c.plain_ffn);
        for (const auto& t : model.tensors) {
            int role = -1, layer = -1;
            if (!neon_cuda::tensor_role(t.name, &role, &layer)) role = -1;
            std::printf("%s %d %d %llu %llu %d %zu\n", t.name.c_str(), role, layer,
                        (unsigned long long)t.shape[0], (unsigned long long)(t.shape.size() > 1 ? t.shape[1] : 0),
                        static_cast<int>(t.type), t.nbytes);
        }
        return 0;
    } catch (const std::exception& e) {
        std::printf("error %s\n", e.what());
        return 1;
    }
}
