// libopworks_llama.so: the C ABI of include/opworks_llama.h over
// include/models/llama.cuh.
//
// No exception crosses the ABI. A failing call records its message (per
// thread, readable with opw_llama_last_error), copies it into the caller's
// `err` buffer when one is given, and returns its failure value: -1 or NULL.
// That is the contract of OpWorks src/llama_c_api.cu:16-35; the code below is
// this library's own.

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <exception>
#include <memory>
#include <string>
#include <type_traits>
#include <variant>
#include <vector>

#include "models/llama.cuh"
#include "opworks_llama.h"

namespace {

// ------------------------------------------------------------ failures

std::string &last_message() {
    thread_local std::string text;
    return text;
}

void report_failure(const char *text, char *buf, int cap) {
    std::string &m = last_message();
    m = text ? text : "unknown error";
    if (buf && cap > 0) {
        const size_t n = std::min(m.size(), static_cast<size_t>(cap) - 1);
        std::memcpy(buf, m.data(), n);
        buf[n] = '\0';
    }
}

// Runs `body` and returns its value; if it throws, reports the failure and
// returns `on_failure` instead.
template <typename R, typename Body> R shielded(R on_failure, char *err, int err_len, Body &&body) noexcept {
    try {
        return body();
    } catch (const std::exception &e) {
        report_failure(e.what(), err, err_len);
    } catch (...) {
        report_failure("unknown C++ exception", err, err_len);
    }
    return on_failure;
}

template <typename H> H &deref(void *handle, const char *what) {
    if (!handle)
        throw std::invalid_argument(std::string("null ") + what);
    return *static_cast<H *>(handle);
}

// ------------------------------------------------------------ handles

// A loaded pack: the fp32 (LlamaModel) or the bf16 (LlamaModelBF16) build of
// the model, chosen by the pack's dtype.
class ModelHandle {
  public:
    template <typename M> explicit ModelHandle(M &&m) : model_(std::forward<M>(m)) {}

    template <typename F> decltype(auto) visit(F &&f) { return std::visit(std::forward<F>(f), model_); }
    int device() {
        return visit([](auto &m) { return m.device(); });
    }
    // Makes the model's device current on the calling thread.
    void activate() { OPWORKS_CUDA_CHECK(cudaSetDevice(device())); }

    static ModelHandle *open(const char *pack_path, unsigned sets, int max_positions) {
        if (!pack_path)
            throw std::invalid_argument("null pack path");
        const std::string dtype = opworks::PackReader(pack_path).dtype();
        if (dtype == "float32")
            return new ModelHandle(opworks::LlamaModel::load(pack_path, sets, max_positions));
        if (dtype == "bfloat16")
            return new ModelHandle(opworks::LlamaModelBF16::load(pack_path, sets, max_positions));
        throw std::runtime_error("unsupported pack dtype " + dtype);
    }

  private:
    std::variant<opworks::LlamaModel, opworks::LlamaModelBF16> model_;
};

// A single-sequence session (the reference's object). It keeps a raw pointer
// to its model, as OpWorks does: sessions are destroyed before their model.
class SessionHandle {
  public:
    template <typename S> SessionHandle(ModelHandle *m, S &&s) : model(m), state_(std::forward<S>(s)) {}

    // f(model, session) on the matching model build.
    template <typename F> decltype(auto) run(F &&f) {
        return model->visit([&](auto &m) -> decltype(auto) {
            using Session = typename std::decay_t<decltype(m)>::Session;
            return f(m, std::get<Session>(state_));
        });
    }

    ModelHandle *const model;

  private:
    std::variant<opworks::LlamaModel::Session, opworks::LlamaModelBF16::Session> state_;
};

// A batched engine over one model (same lifetime rule as a session).
class BatchHandle {
  public:
    explicit BatchHandle(ModelHandle *m) : model(m) {}

    template <typename F> decltype(auto) run(F &&f) {
        return std::visit([&](auto &e) -> decltype(auto) { return f(*e); }, engine_);
    }
    // Builds the engine from the model (`make(model)` returns a unique_ptr).
    template <typename Make> void build(Make &&make) {
        model->visit([&](auto &m) { engine_ = make(m); });
    }

    ModelHandle *const model;

  private:
    std::variant<std::unique_ptr<opworks::LlamaEngineT<float>>,
                 std::unique_ptr<opworks::LlamaEngineT<__nv_bfloat16>>>
        engine_;
};

opworks::SampleArgs sample_args(int i, const float *temperature, const float *top_p, const double *uniforms,
                                const uint64_t *seeds, const int32_t *steps) {
    opworks::SampleArgs sa;
    sa.temperature = temperature ? temperature[i] : 0.f;
    sa.top_p = top_p ? top_p[i] : 1.f;
    sa.uniform = uniforms ? uniforms[i] : -1.0;
    sa.seed = seeds ? seeds[i] : 0;
    sa.step = steps ? steps[i] : 0;
    return sa;
}

} // namespace

extern "C" {

// ------------------------------------------------------------ OpWorks ABI

void *opw_llama_load(const char *pack_path, char *err, int err_len) {
    return shielded<void *>(nullptr, err, err_len, [&] { return ModelHandle::open(pack_path, 0, 8192); });
}

void opw_llama_free(void *model) {
    if (!model)
        return;
    auto *m = static_cast<ModelHandle *>(model);
    cudaSetDevice(m->device());
    delete m;
}

void *opw_llama_create_session(void *model, int max_seq_len, char *err, int err_len) {
    return shielded<void *>(nullptr, err, err_len, [&]() -> void * {
        auto &m = deref<ModelHandle>(model, "model");
        m.activate();
        return m.visit([&](auto &md) { return new SessionHandle(&m, md.create_session(max_seq_len)); });
    });
}

void opw_llama_destroy_session(void *session) {
    if (!session)
        return;
    auto *s = static_cast<SessionHandle *>(session);
    cudaSetDevice(s->model->device());
    delete s;
}

int opw_llama_reset_session(void *session, char *err, int err_len) {
    return shielded(-1, err, err_len, [&] {
        auto &s = deref<SessionHandle>(session, "session");
        s.model->activate();
        s.run([](auto &, auto &sess) { sess.cache.reset(); });
        return 0;
    });
}

int opw_llama_prefill(void *session, const int32_t *tokens, int n, char *err, int err_len) {
    return shielded(-1, err, err_len, [&] {
        auto &s = deref<SessionHandle>(session, "session");
        if (n < 0)
            throw std::invalid_argument("negative token count");
        if (!tokens && n > 0)
            throw std::invalid_argument("null token buffer");
        s.model->activate();
        const std::vector<int32_t> ids(tokens, tokens + n);
        return static_cast<int>(s.run([&](auto &m, auto &sess) { return m.prefill(sess, ids); }));
    });
}

int opw_llama_decode_step(void *session, int32_t prev_token, char *err, int err_len) {
    return shielded(-1, err, err_len, [&] {
        auto &s = deref<SessionHandle>(session, "session");
        s.model->activate();
        return static_cast<int>(s.run([&](auto &m, auto &sess) { return m.decode_step(sess, prev_token); }));
    });
}

int opw_llama_is_eos(void *session, int32_t token, char *err, int err_len) {
    return shielded(-1, err, err_len, [&] {
        auto &s = deref<SessionHandle>(session, "session");
        return s.model->visit([&](auto &m) { return m.is_eos(token) ? 1 : 0; });
    });
}

int opw_llama_last_logits(void *session, float *out, int n, char *err, int err_len) {
    return shielded(-1, err, err_len, [&] {
        auto &s = deref<SessionHandle>(session, "session");
        if (!out)
            throw std::invalid_argument("null logits buffer");
        s.model->activate();
        s.run([&](auto &m, auto &sess) { m.copy_last_logits(sess, out, n); });
        return 0;
    });
}

// Not guarded, as in OpWorks (src/llama_c_api.cu:152-155): a NULL session is
// the caller's error.
int opw_llama_vocab_size(void *session) {
    return static_cast<SessionHandle *>(session)->model->visit([](auto &m) { return m.config().vocab_size; });
}

const char *opw_llama_last_error(void) { return last_message().c_str(); }

// ------------------------------------------------------------ extensions

int opw_llama_set_device(int device) {
    return shielded(-1, nullptr, 0, [&] {
        int count = 0;
        OPWORKS_CUDA_CHECK(cudaGetDeviceCount(&count));
        if (device < 0 || device >= count)
            throw std::invalid_argument("device index out of range");
        OPWORKS_CUDA_CHECK(cudaSetDevice(device));
        return 0;
    });
}

void *opw_llama_load_ex(const char *pack_path, unsigned weight_sets, int max_positions, char *err, int err_len) {
    return shielded<void *>(nullptr, err, err_len, [&] {
        if (max_positions <= 0)
            throw std::invalid_argument("max_positions must be positive");
        return ModelHandle::open(pack_path, weight_sets, max_positions);
    });
}

int opw_llama_model_info(void *model, int32_t *out8, char *err, int err_len) {
    return shielded(-1, err, err_len, [&] {
        auto &m = deref<ModelHandle>(model, "model");
        if (!out8)
            throw std::invalid_argument("null output");
        m.visit([&](auto &md) {
            const auto &c = md.config();
            const int32_t v[8] = {c.num_layers, c.hidden_size,  c.intermediate_size, c.num_q_heads,
                                  c.num_kv_heads, c.head_dim, c.vocab_size,        md.device()};
            std::copy(v, v + 8, out8);
        });
        return 0;
    });
}

void *opw_llama_create_batch(void *model, int max_batch, int max_seq_len, int precision, int prefill_rows, char *err,
                             int err_len) {
    return shielded<void *>(nullptr, err, err_len, [&] {
        auto &m = deref<ModelHandle>(model, "model");
        if (precision != 0 && precision != 1)
            throw std::invalid_argument("precision must be 0 (accurate) or 1 (fast)");
        m.activate();
        auto b = std::make_unique<BatchHandle>(&m);
        b->build([&](auto &md) {
            return md.create_engine(max_batch, max_seq_len, static_cast<opworks::Precision>(precision), prefill_rows);
        });
        return b.release();
    });
}

int opw_llama_nccl_unique_id(char *out, char *err, int err_len) {
    return shielded(-1, err, err_len, [&] {
        if (!out)
            throw std::invalid_argument("null output");
        opworks::NcclLite::get().unique_id(out);
        return 0;
    });
}

void *opw_llama_create_batch_tp(void *model, int max_batch, int max_seq_len, int prefill_rows, int tp_rank,
                                int tp_world, const char *nccl_id, char *err, int err_len) {
    return shielded<void *>(nullptr, err, err_len, [&] {
        auto &m = deref<ModelHandle>(model, "model");
        if (!nccl_id)
            throw std::invalid_argument("null NCCL id");
        m.activate();
        opworks::TensorParallel tp;
        tp.rank = tp_rank;
        tp.world = tp_world;
        tp.nccl_id = nccl_id;
        auto b = std::make_unique<BatchHandle>(&m);
        b->build([&](auto &md) {
            return md.create_engine(max_batch, max_seq_len, opworks::Precision::kFast, prefill_rows, tp);
        });
        return b.release();
    });
}

int opw_llama_batch_tp_ipc_handle(void *batch, char *out128, char *err, int err_len) {
    return shielded(-1, err, err_len, [&] {
        auto &b = deref<BatchHandle>(batch, "batch");
        if (!out128)
            throw std::invalid_argument("null output");
        b.model->activate();
        b.run([&](auto &e) { e.tp_ipc_handles(out128); });
        return 0;
    });
}

int opw_llama_batch_tp_open_peers(void *batch, const char *handles, char *err, int err_len) {
    return shielded(-1, err, err_len, [&] {
        auto &b = deref<BatchHandle>(batch, "batch");
        if (!handles)
            throw std::invalid_argument("null handles");
        b.model->activate();
        b.run([&](auto &e) { e.tp_open_peers(handles); });
        return 0;
    });
}

void opw_llama_destroy_batch(void *batch) {
    if (!batch)
        return;
    auto *b = static_cast<BatchHandle *>(batch);
    cudaSetDevice(b->model->device());
    delete b;
}

int opw_llama_batch_reset(void *batch, int slot, char *err, int err_len) {
    return shielded(-1, err, err_len, [&] {
        auto &b = deref<BatchHandle>(batch, "batch");
        b.model->activate();
        b.run([&](auto &e) { e.reset(slot); });
        return 0;
    });
}

int opw_llama_batch_length(void *batch, int slot) {
    return shielded(-1, nullptr, 0, [&] {
        return deref<BatchHandle>(batch, "batch").run([&](auto &e) { return e.length(slot); });
    });
}

int opw_llama_batch_prefill(void *batch, int slot, const int32_t *tokens, int n, float temperature, float top_p,
                            double uniform, uint64_t seed, char *err, int err_len) {
    return shielded(-1, err, err_len, [&] {
        auto &b = deref<BatchHandle>(batch, "batch");
        if (!tokens && n > 0)
            throw std::invalid_argument("null token buffer");
        b.model->activate();
        const opworks::SampleArgs sa = sample_args(0, &temperature, &top_p, &uniform, &seed, nullptr);
        return static_cast<int>(b.run([&](auto &e) { return e.prefill(slot, tokens, n, sa); }));
    });
}

int opw_llama_batch_decode(void *batch, int n, const int32_t *slots, const int32_t *prev_tokens,
                           const float *temperature, const float *top_p, const double *uniforms,
                           const uint64_t *seeds, const int32_t *steps, int32_t *out_tokens, char *err, int err_len) {
    return shielded(-1, err, err_len, [&] {
        auto &b = deref<BatchHandle>(batch, "batch");
        if (n <= 0 || !slots || !prev_tokens || !out_tokens)
            throw std::invalid_argument("decode needs n > 0, slots, prev_tokens and out_tokens");
        b.model->activate();
        std::vector<opworks::SampleArgs> sa;
        for (int i = 0; i < n; ++i)
            sa.push_back(sample_args(i, temperature, top_p, uniforms, seeds, steps));
        b.run([&](auto &e) { e.decode(n, slots, prev_tokens, sa.data(), out_tokens); });
        return 0;
    });
}

int opw_llama_batch_decode_multi(void *batch, int n, const int32_t *slots, const int32_t *prev_tokens,
                                 const float *temperature, const float *top_p, const double *uniforms,
                                 const uint64_t *seeds, const int32_t *steps0, int steps, int eos_id,
                                 int32_t *out_tokens, int32_t *out_counts, char *err, int err_len) {
    return shielded(-1, err, err_len, [&] {
        auto &b = deref<BatchHandle>(batch, "batch");
        if (n <= 0 || steps <= 0 || !slots || !prev_tokens || !out_tokens || !out_counts)
            throw std::invalid_argument("multi-step decode needs n > 0, steps > 0, slots, prev_tokens and outputs");
        b.model->activate();
        std::vector<opworks::SampleArgs> sa;
        for (int i = 0; i < n; ++i)
            sa.push_back(sample_args(i, temperature, top_p, uniforms, seeds, steps0));
        b.run([&](auto &e) {
            e.decode_multi(n, slots, prev_tokens, sa.data(), steps, uniforms, eos_id, out_tokens, out_counts);
        });
        return 0;
    });
}

int opw_llama_batch_logits(void *batch, int row, float *out, int n, char *err, int err_len) {
    return shielded(-1, err, err_len, [&] {
        auto &b = deref<BatchHandle>(batch, "batch");
        if (!out)
            throw std::invalid_argument("null logits buffer");
        b.model->activate();
        b.run([&](auto &e) { e.copy_logits(row, out, n); });
        return 0;
    });
}

int opw_llama_tp_shard(const int32_t *cfg5, int rank, int world, int64_t *out12, char *err, int err_len) {
    return shielded(-1, err, err_len, [&] {
        if (!cfg5 || !out12)
            throw std::invalid_argument("null argument");
        opworks::ModelConfig c;
        c.hidden_size = cfg5[0];
        c.intermediate_size = cfg5[1];
        c.num_q_heads = cfg5[2];
        c.num_kv_heads = cfg5[3];
        c.head_dim = cfg5[4];
        if (c.hidden_size <= 0 || c.intermediate_size <= 0 || c.num_q_heads <= 0 || c.num_kv_heads <= 0 ||
            c.head_dim <= 0)
            throw std::invalid_argument("model dimensions must be positive");
        const opworks::TpShard sh = opworks::tp_shard(c, rank, world);
        const int64_t v[12] = {sh.q_heads, sh.kv_heads, sh.inter,  sh.q_row0, sh.k_row0,  sh.v_row0,
                               sh.q_rows,  sh.kv_rows,  sh.o_col0, sh.gu_row0, sh.gu_rows, sh.down_col0};
        std::copy(v, v + 12, out12);
        return 0;
    });
}

int opw_llama_batch_kv_blocks(void *batch, int slot, int32_t *out, int cap, char *err, int err_len) {
    return shielded(-1, err, err_len, [&] {
        auto &b = deref<BatchHandle>(batch, "batch");
        if (!out && cap > 0)
            throw std::invalid_argument("null output");
        b.model->activate();
        return b.run([&](auto &e) { return e.kv_blocks(slot, out, cap); });
    });
}

int opw_llama_batch_kv_read(void *batch, int slot, int layer, int pos0, int n, float *k_out, float *v_out, char *err,
                            int err_len) {
    return shielded(-1, err, err_len, [&] {
        auto &b = deref<BatchHandle>(batch, "batch");
        if ((!k_out || !v_out) && n > 0)
            throw std::invalid_argument("null output");
        b.model->activate();
        b.run([&](auto &e) { e.read_kv(slot, layer, pos0, n, k_out, v_out); });
        return 0;
    });
}

int opw_llama_batch_kv_pool(void *batch, int layer, int block0, int nblocks, float *k_out, float *v_out, char *err,
                            int err_len) {
    return shielded(-1, err, err_len, [&] {
        auto &b = deref<BatchHandle>(batch, "batch");
        if ((!k_out || !v_out) && nblocks > 0)
            throw std::invalid_argument("null output");
        b.model->activate();
        return b.run([&](auto &e) { return e.read_kv_pool(layer, block0, nblocks, k_out, v_out); });
    });
}

void *opw_llama_batch_stream(void *batch) {
    return shielded<void *>(nullptr, nullptr, 0, [&] {
        return deref<BatchHandle>(batch, "batch").run([](auto &e) { return static_cast<void *>(e.stream()); });
    });
}

int opw_llama_batch_io_bytes(void *batch, int n, int64_t *out2) {
    return shielded(-1, nullptr, 0, [&] {
        auto &b = deref<BatchHandle>(batch, "batch");
        if (!out2)
            throw std::invalid_argument("null output");
        b.run([&](auto &e) {
            out2[0] = e.decode_h2d_bytes();
            out2[1] = e.decode_d2h_bytes(n);
        });
        return 0;
    });
}

int opw_llama_batch_profile(void *batch, int n, int iters, float *ms_per_step, int32_t *launches_per_step,
                            char *labels, int max_kernels, char *err, int err_len) {
    return shielded(-1, err, err_len, [&] {
        auto &b = deref<BatchHandle>(batch, "batch");
        if (!ms_per_step || !launches_per_step || !labels)
            throw std::invalid_argument("null argument");
        b.model->activate();
        return b.run([&](auto &e) {
            const auto times = e.profile_decode(n, iters);
            const int count = std::min<int>(max_kernels, static_cast<int>(times.size()));
            for (int i = 0; i < count; ++i) {
                ms_per_step[i] = static_cast<float>(times[i].ms_per_step);
                launches_per_step[i] = times[i].launches_per_step;
                std::strncpy(labels + 32 * i, times[i].label.c_str(), 31);
                labels[32 * i + 31] = '\0';
            }
            return count;
        });
    });
}

} // extern "C"
