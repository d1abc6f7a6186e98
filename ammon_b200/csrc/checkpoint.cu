// llama2.c checkpoint loader: real weights for the Llama-shaped decode model.
//
// The file layout is llama2.c's (run.c): seven little-endian int32 -- dim, hidden_dim,
// n_layers, n_heads, n_kv_heads, vocab_size, seq_len; a negative vocab_size marks a
// classifier of its own, a positive one a classifier shared with the embedding -- followed by
// fp32 tensors in this order, every matrix row-major [out, in] (the layout the kernels read):
//   token embedding [vocab, dim], rms_att [layers, dim], wq [layers, dim, dim],
//   wk [layers, kv_dim, dim], wv [layers, kv_dim, dim], wo [layers, dim, dim],
//   rms_ffn [layers, dim], w1 [layers, hidden, dim], w2 [layers, dim, hidden],
//   w3 [layers, hidden, dim], rms_final [dim], two RoPE tables [seq, head / 2] each (unused:
//   the kernels compute the rotation), classifier [vocab, dim] when not shared.
// The reference leaves checkpoints to architecture crates (README.md:5,21); this loader is
// the model assembly the benchmark's llama2.c-shaped configs correspond to.
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "internal.h"
#include "ops.h"

namespace ab {

namespace {

struct File {
    FILE* f = nullptr;
    explicit File(const char* path) : f(std::fopen(path, "rb")) {}
    ~File() {
        if (f) std::fclose(f);
    }
};

struct Llama2cLayout {
    ab_llama_config cfg;
    bool shared;
    uint64_t expected_bytes;
};

Llama2cLayout read_layout(FILE* f, const char* path, uint32_t batch, int32_t dtype,
                          float rope_theta) {
    int32_t h[7];
    if (std::fread(h, sizeof(int32_t), 7, f) != 7)
        invalid(std::string("llama2.c checkpoint ") + path + ": shorter than its header");
    const int32_t dim = h[0], hidden = h[1], layers = h[2], heads = h[3], kv_heads = h[4];
    const int32_t vocab = h[5] < 0 ? -h[5] : h[5], seq = h[6];
    if (dim <= 0 || hidden <= 0 || layers <= 0 || heads <= 0 || kv_heads <= 0 || vocab <= 0 ||
        seq <= 0 || dim % heads || heads % kv_heads)
        invalid(std::string("llama2.c checkpoint ") + path + ": implausible header (dim " +
                std::to_string(dim) + ", hidden " + std::to_string(hidden) + ", layers " +
                std::to_string(layers) + ", heads " + std::to_string(heads) + "/" +
                std::to_string(kv_heads) + ", vocab " + std::to_string(h[5]) + ", seq " +
                std::to_string(seq) + ")");
    Llama2cLayout L;
    L.shared = h[5] > 0;
    const uint64_t head = (uint64_t)dim / heads, kvd = head * kv_heads, D = dim, F = hidden;
    const uint64_t per_layer = 2 * D + D * D + 2 * kvd * D + D * D + 3 * F * D;
    const uint64_t floats = (uint64_t)vocab * D + layers * per_layer + D + (uint64_t)seq * head +
                            (L.shared ? 0 : (uint64_t)vocab * D);
    L.expected_bytes = 7 * 4 + floats * 4;
    L.cfg = {};
    L.cfg.dim = (uint32_t)dim;
    L.cfg.layers = (uint32_t)layers;
    L.cfg.heads = (uint32_t)heads;
    L.cfg.kv_heads = (uint32_t)kv_heads;
    L.cfg.head_dim = (uint32_t)head;
    L.cfg.hidden = (uint32_t)hidden;
    L.cfg.vocab = (uint32_t)vocab;
    L.cfg.seq = (uint32_t)seq;
    L.cfg.batch = batch;
    L.cfg.rope_theta = rope_theta;
    L.cfg.norm_eps = 1e-5f;
    L.cfg.dtype = dtype;
    std::fseek(f, 0, SEEK_END);
    const long size = std::ftell(f);
    if (size < 0 || (uint64_t)size != L.expected_bytes)
        invalid(std::string("llama2.c checkpoint ") + path + ": " + std::to_string(size) +
                " bytes, the header's shapes need " + std::to_string(L.expected_bytes));
    std::fseek(f, 7 * 4, SEEK_SET);
    return L;
}

// Round-to-nearest-even fp32 -> bf16 bits (the weights are finite).
inline uint16_t to_bf16_bits(float v) {
    uint32_t u;
    std::memcpy(&u, &v, 4);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

// Throws the status of a failed C entry point, with its last error.
void check(int status) {
    if (status != AB_OK) fail(status, ab_last_error());
}

// Reads `count` fp32 values of the checkpoint into `buf`.
void read_floats(FILE* f, std::vector<float>& buf, uint64_t count, const char* what) {
    buf.resize(count);
    if (std::fread(buf.data(), sizeof(float), count, f) != count)
        invalid(std::string("llama2.c checkpoint: short read of ") + what);
}

// Copies the slice rows [r0, r0 + dst.rows) x cols [c0, c0 + dst.cols) of a row-major host
// matrix [rows, cols] into the device tensor `dst` ([dst rows, dst cols] or a vector),
// converting to the tensor's element type.
void upload(const ab_tensor& dst, const std::vector<float>& src, uint64_t cols, uint64_t r0,
            uint64_t c0) {
    const uint64_t dr = dst.rank == 2 ? dst.dims[0] : 1;
    const uint64_t dc = dst.rank == 2 ? dst.dims[1] : dst.dims[0];
    const size_t esz = dtype_size(dst.dtype);
    std::vector<unsigned char> tmp(dr * dc * esz);
    for (uint64_t r = 0; r < dr; r++) {
        const float* s = src.data() + (r0 + r) * cols + c0;
        if (dst.dtype == AB_F32) {
            std::memcpy(tmp.data() + r * dc * 4, s, dc * 4);
        } else {
            uint16_t* d = reinterpret_cast<uint16_t*>(tmp.data()) + r * dc;
            for (uint64_t c = 0; c < dc; c++) d[c] = to_bf16_bits(s[c]);
        }
    }
    cuda_check(cudaMemcpy(dst.data, tmp.data(), tmp.size(), cudaMemcpyHostToDevice),
               "checkpoint upload");
}

}  // namespace

}  // namespace ab

using namespace ab;

extern "C" {

int ab_llama2c_config(const char* path, uint32_t batch, int32_t dtype, float rope_theta,
                      ab_llama_config* cfg) {
    return guard([&] {
        if (!path || !cfg) fail(AB_ERR_ARGUMENT, "null argument");
        File f(path);
        if (!f.f) invalid(std::string("cannot open llama2.c checkpoint ") + path);
        *cfg = read_layout(f.f, path, batch, dtype, rope_theta).cfg;
    });
}

int ab_llama_load_llama2c(ab_runtime* rt, const char* path, int32_t dtype, uint32_t batch,
                          float rope_theta, ab_comm* comm, ab_llama_config* cfg_out,
                          ab_llama** out) {
    return guard([&] {
        if (!path || !out) fail(AB_ERR_ARGUMENT, "null argument");
        if (dtype != AB_F32 && dtype != AB_BF16) invalid("dtype must be f32 or bf16");
        File f(path);
        if (!f.f) invalid(std::string("cannot open llama2.c checkpoint ") + path);
        const Llama2cLayout L = read_layout(f.f, path, batch, dtype, rope_theta);
        if (!rt) fail(AB_ERR_ARGUMENT, "null runtime");
        ab_llama* m = nullptr;
        check(comm ? ab_llama_create_tp(rt, &L.cfg, comm, &m) : ab_llama_create(rt, &L.cfg, &m));
        try {
            const ab_llama_config& c = L.cfg;
            const int rank = comm ? comm_rank(comm) : 0, world = comm ? comm_world(comm) : 1;
            const uint64_t D = c.dim, F = c.hidden, V = c.vocab, head = c.head_dim;
            const uint64_t qd = (uint64_t)c.heads * head, kvd = (uint64_t)c.kv_heads * head;
            const uint64_t qd_l = qd / world, kvd_l = kvd / world, F_l = F / world,
                           V_l = V / world;
            rt->activate();
            auto w = [&](int which, uint32_t layer) {
                ab_tensor t;
                check(ab_llama_weight(m, which, layer, &t));
                return t;
            };
            std::vector<float> buf, embed;
            read_floats(f.f, embed, V * D, "token embedding");
            upload(w(0, 0), embed, D, 0, 0);
            // per-layer tensors come grouped by kind, every layer in turn
            auto each_layer = [&](const char* what, uint64_t rows, uint64_t cols, int which,
                                  uint64_t r0, uint64_t c0) {
                for (uint32_t l = 0; l < c.layers; l++) {
                    read_floats(f.f, buf, rows * cols, what);
                    upload(w(which, l), buf, cols, r0, c0);
                }
            };
            each_layer("rms_att", 1, D, 3, 0, 0);
            each_layer("wq", qd, D, 4, rank * qd_l, 0);
            each_layer("wk", kvd, D, 5, rank * kvd_l, 0);
            each_layer("wv", kvd, D, 6, rank * kvd_l, 0);
            each_layer("wo", D, qd, 7, 0, rank * qd_l);
            each_layer("rms_ffn", 1, D, 8, 0, 0);
            each_layer("w1", F, D, 9, rank * F_l, 0);
            each_layer("w2", D, F, 10, 0, rank * F_l);
            each_layer("w3", F, D, 11, rank * F_l, 0);
            read_floats(f.f, buf, D, "rms_final");
            upload(w(2, 0), buf, D, 0, 0);
            // skip the two RoPE tables
            if (std::fseek(f.f, (long)(c.seq * head * 4), SEEK_CUR) != 0)
                invalid("llama2.c checkpoint: cannot skip the RoPE tables");
            if (L.shared) {
                upload(w(1, 0), embed, D, rank * V_l, 0);
            } else {
                read_floats(f.f, buf, V * D, "classifier");
                upload(w(1, 0), buf, D, rank * V_l, 0);
            }
            cuda_check(cudaDeviceSynchronize(), "checkpoint upload");
        } catch (...) {
            ab_llama_destroy(m);
            throw;
        }
        if (cfg_out) *cfg_out = L.cfg;
        *out = m;
    });
}

}  // extern "C"
