// Exercises the C++ drop-in the way the reference's code calls it:
// flash_attention_forward(Q, K, V, scale, true) (OlmoAttention.cpp:94) and an
// OlmoBlock-like owner holding OlmoAttention by value (OlmoBlock.h:19) that
// constructs it from (folder, index) and calls forward (OlmoBlock.cpp:6,14).
//
//   test_dropin flash <dir> B T H     reads dir/{q,k,v,do}.f32, writes dir/{o,m,l}.f32 and
//                                     flash_attention_backward's dir/{dq,dk,dv}.f32
//   test_dropin layer <dir> index B T reads dir/x.f32 and the layer's .npy weights
//                                     from dir, writes dir/y.f32
//   test_dropin train <dir> index B T reads dir/{x,dy}.f32: forward, backward (writes dir/dx.f32),
//                                     step(1e-3), forward again (writes dir/y2.f32), zero_grad
//                                     -- the OlmoBlock calls (OlmoBlock.cpp:14,28,33,40)
//   test_dropin tokens <dir> <vocab> <file>...  token_batch of the files padded with the
//                                     vocab's <|pad|> id (main.cpp:14-58): writes
//                                     dir/batch.u32, prints "rows cols pad"
//   test_dropin model <dir> L B T     reads dir/ids.u32 and an L-layer checkpoint from
//                                     dir, writes dir/logits.f32 (OlmoModel)
//   test_dropin layer_tp <dir> index B T world rank
//                                     head-parallel: rank 0 writes the NCCL id to
//                                     dir/nccl.id, every rank (GPU = rank) makes its
//                                     communicator, calls set_tensor_parallel, runs the
//                                     BlockLike forward on dir/x.f32 and writes dir/y<rank>.f32
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <iostream>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "FlashAttention.h"
#include "OlmoAttention.h"
#include "OlmoModel.h"
#include "Tokens.h"
#include "dirktensor_b200.h"

template <class X>
static void read_into(const std::string& path, X& x) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("cannot open " + path);
    f.read(reinterpret_cast<char*>(x.data()), static_cast<std::streamsize>(x.size() * sizeof(float)));
}

template <class X>
static void write_from(const std::string& path, const X& x) {
    std::ofstream f(path, std::ios::binary);
    f.write(reinterpret_cast<const char*>(x.data()), static_cast<std::streamsize>(x.size() * sizeof(float)));
}

struct BlockLike {
    OlmoAttention m_attention;
    BlockLike(const std::string& folder, unsigned index) : m_attention(folder, index) {}
    xt::xtensor<float, 3> forward(const xt::xtensor<float, 3>& x) { return m_attention.forward(x); }
    xt::xtensor<float, 3> backward(const xt::xtensor<float, 3>& d) { return m_attention.backward(d); }
    void step(float lr) { m_attention.step(lr); }
    void zero_grad() { m_attention.zero_grad(); }
};

int main(int argc, char** argv) {
    try {
        if (argc < 3) throw std::runtime_error("usage: test_dropin flash|layer <dir> ...");
        const std::string mode = argv[1], dir = argv[2];
        if (mode == "flash" && argc == 6) {
            const std::size_t B = std::stoul(argv[3]), T = std::stoul(argv[4]), H = std::stoul(argv[5]);
            xt::xtensor<float, 4> q = xt::empty<float>({B, T, H, std::size_t(128)});
            xt::xtensor<float, 4> k = xt::empty<float>({B, T, H, std::size_t(128)});
            xt::xtensor<float, 4> v = xt::empty<float>({B, T, H, std::size_t(128)});
            read_into(dir + "/q.f32", q);
            read_into(dir + "/k.f32", k);
            read_into(dir + "/v.f32", v);
            const FlashAttentionResult r = flash_attention_forward(q, k, v, 1.0f / 11.313708498984761f, true);
            write_from(dir + "/o.f32", r.output);
            write_from(dir + "/m.f32", r.softmax_m);
            write_from(dir + "/l.f32", r.softmax_l);
            xt::xtensor<float, 4> d_out = xt::empty<float>({B, T, H, std::size_t(128)});
            read_into(dir + "/do.f32", d_out);
            const FlashAttentionGradients g = flash_attention_backward(d_out, r.output, r.softmax_m, r.softmax_l, q,
                                                                       k, v, 1.0f / 11.313708498984761f, true);
            write_from(dir + "/dq.f32", g.d_Q);
            write_from(dir + "/dk.f32", g.d_K);
            write_from(dir + "/dv.f32", g.d_V);
        } else if (mode == "layer" && argc == 6) {
            const unsigned index = static_cast<unsigned>(std::stoul(argv[3]));
            const std::size_t B = std::stoul(argv[4]), T = std::stoul(argv[5]);
            xt::xtensor<float, 3> x = xt::empty<float>({B, T, std::size_t(2048)});
            read_into(dir + "/x.f32", x);
            BlockLike block(dir, index);
            BlockLike moved(std::move(block));  // the class is move-only
            const xt::xtensor<float, 3> y = moved.forward(x);
            write_from(dir + "/y.f32", y);
            moved.m_attention.zero_grad();
        } else if (mode == "train" && argc == 6) {
            const unsigned index = static_cast<unsigned>(std::stoul(argv[3]));
            const std::size_t B = std::stoul(argv[4]), T = std::stoul(argv[5]);
            xt::xtensor<float, 3> x = xt::empty<float>({B, T, std::size_t(2048)});
            xt::xtensor<float, 3> dy = xt::empty<float>({B, T, std::size_t(2048)});
            read_into(dir + "/x.f32", x);
            read_into(dir + "/dy.f32", dy);
            BlockLike block(dir, index);
            block.forward(x);
            write_from(dir + "/dx.f32", block.backward(dy));
            block.step(1e-3f);
            write_from(dir + "/y2.f32", block.forward(x));
            block.zero_grad();
        } else if (mode == "layer_tp" && argc == 8) {
            const unsigned index = static_cast<unsigned>(std::stoul(argv[3]));
            const std::size_t B = std::stoul(argv[4]), T = std::stoul(argv[5]);
            const int world = std::stoi(argv[6]), rank = std::stoi(argv[7]);
            unsigned char id[128];
            const std::string idf = dir + "/nccl.id";
            if (rank == 0) {
                if (dt_comm_unique_id(id) != DT_OK) throw std::runtime_error(dt_last_error());
                std::ofstream(idf + ".tmp", std::ios::binary).write(reinterpret_cast<const char*>(id), 128);
                std::rename((idf + ".tmp").c_str(), idf.c_str());
            } else {
                for (int i = 0;; ++i) {  // bounded wait for rank 0's id
                    std::ifstream f(idf, std::ios::binary);
                    if (f && f.read(reinterpret_cast<char*>(id), 128)) break;
                    if (i > 600) throw std::runtime_error("no NCCL id from rank 0");
                    std::this_thread::sleep_for(std::chrono::milliseconds(100));
                }
            }
            dt_comm* comm = nullptr;
            if (dt_comm_create(id, world, rank, rank, 60000, &comm) != DT_OK) throw std::runtime_error(dt_last_error());
            dirktensor_b200::set_tensor_parallel(comm);
            {
                xt::xtensor<float, 3> x = xt::empty<float>({B, T, std::size_t(2048)});
                read_into(dir + "/x.f32", x);
                BlockLike block(dir, index);
                const xt::xtensor<float, 3> y = block.forward(x);
                write_from(dir + "/y" + std::to_string(rank) + ".f32", y);
                try {  // training stays single-GPU
                    block.backward(y);
                    return 4;
                } catch (const std::runtime_error&) {
                }
            }
            dirktensor_b200::set_tensor_parallel(nullptr);
            if (dt_comm_destroy(comm) != DT_OK) throw std::runtime_error(dt_last_error());
        } else if (mode == "tokens" && argc >= 5) {
            const uint32_t pad = pad_token_id(argv[3]);
            std::vector<std::string> files(argv + 4, argv + argc);
            const xt::xtensor<uint32_t, 2> batch = token_batch(files, pad);
            std::ofstream f(dir + "/batch.u32", std::ios::binary);
            f.write(reinterpret_cast<const char*>(batch.data()), static_cast<std::streamsize>(batch.size() * 4));
            std::cout << batch.shape(0) << " " << batch.shape(1) << " " << pad << "\n";
        } else if (mode == "model" && argc == 6) {
            const unsigned layers = static_cast<unsigned>(std::stoul(argv[3]));
            const std::size_t B = std::stoul(argv[4]), T = std::stoul(argv[5]);
            xt::xtensor<uint32_t, 2> ids = xt::empty<uint32_t>({B, T});
            std::ifstream f(dir + "/ids.u32", std::ios::binary);
            f.read(reinterpret_cast<char*>(ids.data()), static_cast<std::streamsize>(ids.size() * 4));
            OlmoModel model(dir, layers);
            const xt::xtensor<float, 3> logits = model.forward(ids);
            write_from(dir + "/logits.f32", logits);
            try {
                model.step(1e-4f);
                return 3;
            } catch (const std::logic_error&) {
            }
        } else {
            throw std::runtime_error("bad arguments");
        }
    } catch (const std::exception& e) {
        std::cerr << "error: " << e.what() << "\n";
        return 1;
    }
    return 0;
}
