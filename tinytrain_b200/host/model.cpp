// GPTModel on the device: the reference's Llama decoder (model.cpp:14-160 of
// seampm/tinytrain) with its per-op chains replaced by fused device ops:
//   attention block  rmsnorm -> 3 x linear -> causal_attention (RoPE, scale,
//                    causal softmax and P.V in one kernel) -> linear -> add
//   FFN block        rmsnorm -> 2 x linear -> swiglu -> linear -> add
//   head             rmsnorm -> linear against the tied embedding table
// Construction, parameter order, seeds, RoPE tables and checkpoint format are
// the reference's, so a model built here from a seed has the reference's
// weights and its checkpoints load into either implementation.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <map>
#include <sstream>
#include <stdexcept>

#include "internal.h"
#include "nn_init.h"
#include "tinytrain/model.h"
#include "tinytrain/ops.h"

namespace tt {

using namespace detail;

GPTModel::GPTModel(const GPTConfig& cfg, uint64_t seed) : GPTModel(cfg, seed, true) {}

GPTModel::GPTModel(const GPTConfig& cfg, uint64_t seed, bool host_init) : cfg_(cfg) {
    if (cfg.dim % cfg.n_heads != 0)
        throw std::invalid_argument("GPTModel: dim must divide n_heads");
    const int64_t hd = cfg.dim / cfg.n_heads;
    if (hd % 2 != 0)
        throw std::invalid_argument("GPTModel: head_dim must be even");

    HostInitScope scope(host_init);
    tok_embeddings = Embedding(cfg.vocab_size, cfg.dim, seed + 1);
    blocks_.reserve(static_cast<size_t>(cfg.n_layers));
    for (int64_t l = 0; l < cfg.n_layers; ++l) {
        Block b;
        const uint64_t s = seed + 100 + static_cast<uint64_t>(l) * 10;
        b.rms_attn = RMSNorm(cfg.dim, cfg.norm_eps);
        b.wq = Linear(cfg.dim, cfg.n_heads * hd, s + 0);
        b.wk = Linear(cfg.dim, cfg.n_kv_heads * hd, s + 1);
        b.wv = Linear(cfg.dim, cfg.n_kv_heads * hd, s + 2);
        b.wo = Linear(cfg.n_heads * hd, cfg.dim, s + 3);
        b.rms_ffn = RMSNorm(cfg.dim, cfg.norm_eps);
        b.wgate = Linear(cfg.dim, cfg.ffn_dim, s + 4);
        b.wup = Linear(cfg.dim, cfg.ffn_dim, s + 5);
        b.wdown = Linear(cfg.ffn_dim, cfg.dim, s + 6);
        blocks_.push_back(std::move(b));
    }
    rms_final = RMSNorm(cfg.dim, cfg.norm_eps);
    tie_weights_ = true;

    // RoPE tables: cos/sin of pos / theta^(2i/hd) in float (model.cpp:43-53).
    const int64_t Dh = hd / 2;
    std::vector<float> c(static_cast<size_t>(cfg.max_seq_len * Dh)),
        s(static_cast<size_t>(cfg.max_seq_len * Dh));
    for (int64_t pos = 0; pos < cfg.max_seq_len; ++pos)
        for (int64_t i = 0; i < Dh; ++i) {
            const float inv_freq =
                1.0f / std::pow(cfg.rope_theta, (2.0f * i) / static_cast<float>(hd));
            const float angle = static_cast<float>(pos) * inv_freq;
            c[static_cast<size_t>(pos * Dh + i)] = std::cos(angle);
            s[static_cast<size_t>(pos * Dh + i)] = std::sin(angle);
        }
    rope_cos_ = Tensor({cfg.max_seq_len, Dh});
    rope_sin_ = Tensor({cfg.max_seq_len, Dh});
    rope_cos_.copy_from_host(c.data());
    rope_sin_.copy_from_host(s.data());
}

std::vector<Tensor*> GPTModel::parameters() {
    std::vector<Tensor*> ps;
    ps.push_back(&tok_embeddings.weight);
    for (auto& b : blocks_) {
        ps.push_back(&b.rms_attn.weight);
        ps.push_back(&b.wq.weight);
        ps.push_back(&b.wk.weight);
        ps.push_back(&b.wv.weight);
        ps.push_back(&b.wo.weight);
        ps.push_back(&b.rms_ffn.weight);
        ps.push_back(&b.wgate.weight);
        ps.push_back(&b.wup.weight);
        ps.push_back(&b.wdown.weight);
    }
    ps.push_back(&rms_final.weight);
    if (!tie_weights_)
        ps.push_back(&lm_head.weight);
    return ps;
}

void GPTModel::init_normal_(float std, uint64_t seed) {
    uint64_t k = 0;
    for (Tensor* p : parameters()) {
        if (p->ndim() == 1)
            p->impl()->data->fill(1.0f);
        else
            check(ttk_init_normal(p->impl()->data->device_for_overwrite(), p->numel(), std,
                                  seed * 1000003ull + (k++), stream()),
                  "init_normal");
    }
}

Tensor GPTModel::forward(const std::vector<int64_t>& idx, int64_t B, int64_t T) {
    if (static_cast<int64_t>(idx.size()) != B * T)
        throw std::invalid_argument("GPTModel::forward: idx size mismatch");
    if (T > cfg_.max_seq_len)
        throw std::invalid_argument("GPTModel::forward: sequence too long");
    for (int64_t t : idx)
        if (t < 0 || t >= cfg_.vocab_size)
            throw std::invalid_argument("embedding: index out of range");
    return forward(DeviceIds(idx), B, T);
}

Tensor GPTModel::forward(const DeviceIds& idx, int64_t B, int64_t T) {
    if (idx.size() != B * T)
        throw std::invalid_argument("GPTModel::forward: idx size mismatch");
    if (T > cfg_.max_seq_len)
        throw std::invalid_argument("GPTModel::forward: sequence too long");
    const int64_t H = cfg_.n_heads, hd = cfg_.dim / H, R = B * T, d = cfg_.dim;
    const bool drop = cfg_.dropout > 0.0f && training;
    // The fused kernel covers head dims 32/64/128 without dropout; otherwise
    // the reference's op chain runs on device ops.
    const bool fused = !drop && (hd == 32 || hd == 64 || hd == 128);

    Tensor x = embedding(tok_embeddings.weight, idx);  // [R, d]
    for (auto& b : blocks_) {
        Tensor h = rmsnorm(x, b.rms_attn.weight, b.rms_attn.eps);
        Tensor q = reshape(linear(h, b.wq.weight), {B, T, H, hd});
        Tensor k = reshape(linear(h, b.wk.weight), {B, T, H, hd});
        Tensor v = reshape(linear(h, b.wv.weight), {B, T, H, hd});
        Tensor att;
        if (fused) {
            att = causal_attention(q, k, v, rope_cos_, rope_sin_);
        } else {
            // Dropout on the attention probabilities needs them materialized,
            // and other head dims have no fused kernel: the reference's op
            // chain (model.cpp:127-141) on device ops.
            const int64_t Dh = hd / 2;
            Tensor cos = reshape(rope_cos_, {cfg_.max_seq_len, Dh});
            Tensor sin = reshape(rope_sin_, {cfg_.max_seq_len, Dh});
            if (T != cfg_.max_seq_len) {
                std::vector<float> ch(static_cast<size_t>(T * Dh)), sh(static_cast<size_t>(T * Dh));
                std::memcpy(ch.data(), rope_cos_.data(), ch.size() * 4);
                std::memcpy(sh.data(), rope_sin_.data(), sh.size() * 4);
                cos = Tensor({T, Dh});
                sin = Tensor({T, Dh});
                cos.copy_from_host(ch.data());
                sin.copy_from_host(sh.data());
            }
            Tensor mask = full({T, T}, 0.0f);
            std::vector<float> mh(static_cast<size_t>(T * T), 0.0f);
            for (int64_t i = 0; i < T; ++i)
                for (int64_t j = i + 1; j < T; ++j)
                    mh[static_cast<size_t>(i * T + j)] = -1e9f;
            mask.copy_from_host(mh.data());
            const float scale = 1.0f / std::sqrt(static_cast<float>(hd));
            Tensor qb = reshape(permute(rope(q, cos, sin), {0, 2, 1, 3}), {B * H, T, hd});
            Tensor kb = reshape(permute(rope(k, cos, sin), {0, 2, 1, 3}), {B * H, T, hd});
            Tensor vb = reshape(permute(v, {0, 2, 1, 3}), {B * H, T, hd});
            Tensor scores = bmm(qb, transpose(kb, 1, 2));
            scores = add(mul(scores, full(scores.shape(), scale)), mask);
            Tensor probs = softmax(scores, -1);
            if (drop)
                probs = dropout(probs, cfg_.dropout, ++dropout_seed_);
            Tensor a = bmm(probs, vb);
            att = reshape(permute(reshape(a, {B, H, T, hd}), {0, 2, 1, 3}), {B, T, H * hd});
        }
        Tensor att_out = linear(reshape(att, {R, d}), b.wo.weight);
        if (drop)
            att_out = dropout(att_out, cfg_.dropout, ++dropout_seed_);
        x = add(x, att_out);

        Tensor hff = rmsnorm(x, b.rms_ffn.weight, b.rms_ffn.eps);
        Tensor ffn = ffn_swiglu(hff, b.wgate.weight, b.wup.weight, b.wdown.weight);
        if (drop)
            ffn = dropout(ffn, cfg_.dropout, ++dropout_seed_);
        x = add(x, ffn);
    }
    Tensor hn = rmsnorm(x, rms_final.weight, rms_final.eps);
    return linear(hn, tok_embeddings.weight);  // tied head: hn @ E^T
}

// -------------------------------------------------------------- checkpoints --
// safetensors: 8-byte little-endian header length, a JSON header mapping
// tensor names to {dtype, shape, data_offsets}, then the raw LE float32
// payloads (model.cpp:162-227). Written with a small emitter of this exact
// JSON subset and read with a matching scanner.

namespace {

struct Named {
    std::string name;
    Tensor* t;
};

std::vector<Named> checkpoint_tensors(GPTModel& m, const GPTConfig& cfg) {
    auto ps = m.parameters();
    std::vector<Named> out;
    out.push_back({"model.embed_tokens.weight", ps[0]});
    for (int64_t l = 0; l < cfg.n_layers; ++l) {
        const std::string pre = "model.layers." + std::to_string(l);
        Tensor** b = &ps[static_cast<size_t>(1 + 9 * l)];
        out.push_back({pre + ".self_attn.q_proj.weight", b[1]});
        out.push_back({pre + ".self_attn.k_proj.weight", b[2]});
        out.push_back({pre + ".self_attn.v_proj.weight", b[3]});
        out.push_back({pre + ".self_attn.o_proj.weight", b[4]});
        out.push_back({pre + ".mlp.gate_proj.weight", b[6]});
        out.push_back({pre + ".mlp.up_proj.weight", b[7]});
        out.push_back({pre + ".mlp.down_proj.weight", b[8]});
        out.push_back({pre + ".input_layernorm.weight", b[0]});
        out.push_back({pre + ".post_attention_layernorm.weight", b[5]});
    }
    out.push_back({"model.norm.weight", ps[static_cast<size_t>(1 + 9 * cfg.n_layers)]});
    return out;
}

std::string num(double v) {
    char buf[64];
    std::snprintf(buf, sizeof(buf), "%.9g", v);
    return buf;
}

// Finds "key": in `s` starting at `from` and returns the position after ':'.
size_t find_key(const std::string& s, const std::string& key, size_t from) {
    const std::string pat = "\"" + key + "\"";
    size_t p = s.find(pat, from);
    if (p == std::string::npos)
        return p;
    p = s.find(':', p + pat.size());
    return p == std::string::npos ? p : p + 1;
}

}  // namespace

void GPTModel::save_checkpoint(const std::string& dir) const {
    namespace fs = std::filesystem;
    fs::create_directories(dir);
    auto tensors = checkpoint_tensors(const_cast<GPTModel&>(*this), cfg_);
    // Keys sorted like nlohmann::json's object (std::map) so the header
    // matches the reference's byte for byte; payloads in list order.
    std::map<std::string, std::string> entries;
    int64_t offset = 0;
    for (auto& nt : tensors) {
        const int64_t nbytes = nt.t->numel() * 4;
        std::string shape = "[";
        for (size_t i = 0; i < nt.t->shape().size(); ++i)
            shape += (i ? "," : "") + std::to_string(nt.t->shape()[i]);
        shape += "]";
        entries[nt.name] = "{\"data_offsets\":[" + std::to_string(offset) + "," +
                           std::to_string(offset + nbytes) + "],\"dtype\":\"F32\",\"shape\":" +
                           shape + "}";
        offset += nbytes;
    }
    std::string header = "{";
    bool first = true;
    for (auto& [k, v] : entries) {
        header += (first ? "\"" : ",\"") + k + "\":" + v;
        first = false;
    }
    header += "}";
    std::ofstream f(dir + "/model.safetensors", std::ios::binary);
    if (!f)
        throw std::runtime_error("save_checkpoint: cannot open model.safetensors");
    const uint64_t hlen = header.size();
    f.write(reinterpret_cast<const char*>(&hlen), 8);
    f.write(header.data(), static_cast<std::streamsize>(header.size()));
    std::vector<float> buf;
    for (auto& nt : tensors) {
        buf.resize(static_cast<size_t>(nt.t->numel()));
        nt.t->copy_to_host(buf.data());
        f.write(reinterpret_cast<const char*>(buf.data()),
                static_cast<std::streamsize>(nt.t->numel() * 4));
    }
    f.close();
    std::ofstream cf(dir + "/config.json");
    cf << "{\n  \"hidden_size\": " << cfg_.dim << ",\n  \"intermediate_size\": " << cfg_.ffn_dim
       << ",\n  \"max_position_embeddings\": " << cfg_.max_seq_len
       << ",\n  \"num_attention_heads\": " << cfg_.n_heads
       << ",\n  \"num_hidden_layers\": " << cfg_.n_layers
       << ",\n  \"num_key_value_heads\": " << cfg_.n_kv_heads
       << ",\n  \"rms_norm_eps\": " << num(cfg_.norm_eps)
       << ",\n  \"rope_theta\": " << num(cfg_.rope_theta)
       << ",\n  \"vocab_size\": " << cfg_.vocab_size << "\n}";
}

void GPTModel::load_checkpoint(const std::string& dir) {
    const std::string path = dir + "/model.safetensors";
    std::ifstream f(path, std::ios::binary);
    if (!f)
        throw std::runtime_error("load_checkpoint: cannot open " + path);
    uint64_t hlen = 0;
    f.read(reinterpret_cast<char*>(&hlen), 8);
    if (!f || hlen > (1ull << 30))
        throw std::runtime_error("load_checkpoint: bad header");
    std::string hstr(static_cast<size_t>(hlen), '\0');
    f.read(hstr.data(), static_cast<std::streamsize>(hlen));
    auto tensors = checkpoint_tensors(*this, cfg_);
    std::vector<float> buf;
    for (auto& nt : tensors) {
        const std::string key = "\"" + nt.name + "\"";
        const size_t at = hstr.find(key);
        if (at == std::string::npos)
            throw std::runtime_error("load_checkpoint: missing tensor " + nt.name);
        const size_t obj_end = hstr.find('}', at);
        size_t p = find_key(hstr, "data_offsets", at);
        if (p == std::string::npos || p > obj_end)
            throw std::runtime_error("load_checkpoint: missing tensor " + nt.name);
        p = hstr.find('[', p);
        uint64_t beg = 0, end = 0;
        if (std::sscanf(hstr.c_str() + p, "[%lu,%lu]", &beg, &end) != 2)
            throw std::runtime_error("load_checkpoint: bad offsets for " + nt.name);
        if (end - beg != static_cast<uint64_t>(nt.t->numel() * 4))
            throw std::runtime_error("load_checkpoint: size mismatch for " + nt.name);
        buf.resize(static_cast<size_t>(nt.t->numel()));
        f.seekg(static_cast<std::streamoff>(8 + hlen + beg), std::ios::beg);
        f.read(reinterpret_cast<char*>(buf.data()), static_cast<std::streamsize>(nt.t->numel() * 4));
        if (!f)
            throw std::runtime_error("load_checkpoint: read failed for " + nt.name);
        nt.t->copy_from_host(buf.data());
    }
}

}  // namespace tt
