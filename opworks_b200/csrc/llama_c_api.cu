// libopworks_llama.so: the C ABI of include/opworks_llama.h over
// include/models/llama.cuh. Every guarded call turns C++ exceptions into
// -1 / NULL plus an error string (copied into `err` and kept thread-locally),
// matching OpWorks src/llama_c_api.cu:16-35.

#include <cstdint>
#include <cstring>
#include <exception>
#include <memory>
#include <string>
#include <variant>
#include <vector>

#include "models/llama.cuh"
#include "opworks_llama.h"

namespace {

thread_local std::string g_last_error;

int capture_error(const char *what, char *err, int err_len) {
    g_last_error = what ? what : "unknown error";
    if (err && err_len > 0) {
        std::strncpy(err, g_last_error.c_str(), static_cast<size_t>(err_len) - 1);
        err[err_len - 1] = '\0';
    }
    return -1;
}

template <typename F> int guard(F &&f, char *err, int err_len) {
    try {
        return f();
    } catch (const std::exception &e) {
        return capture_error(e.what(), err, err_len);
    } catch (...) {
        return capture_error("unknown C++ exception", err, err_len);
    }
}

template <typename F> void *guard_ptr(F &&f, char *err, int err_len) {
    try {
        return f();
    } catch (const std::exception &e) {
        capture_error(e.what(), err, err_len);
    } catch (...) {
        capture_error("unknown C++ exception", err, err_len);
    }
    return nullptr;
}

using ModelVariant = std::variant<opworks::LlamaModel, opworks::LlamaModelBF16>;

struct ModelHolder {
    ModelVariant model;
};

template <typename F> auto with_model(ModelHolder *m, F &&f) {
    return std::visit([&](auto &model) { return f(model); }, m->model);
}

// A session is the reference's single-sequence object (owner back-pointer,
// as in OpWorks: sessions must be destroyed before their model).
struct SessionHolder {
    ModelHolder *owner;
    std::variant<opworks::LlamaModel::Session, opworks::LlamaModelBF16::Session> session;
};

struct BatchHolder {
    ModelHolder *owner;
    std::variant<std::unique_ptr<opworks::LlamaEngineT<float>>, std::unique_ptr<opworks::LlamaEngineT<__nv_bfloat16>>>
        engine;
};

template <typename F> auto with_session(SessionHolder *s, F &&f) {
    return std::visit(
        [&](auto &model) {
            using M = std::decay_t<decltype(model)>;
            auto &sess = std::get<typename M::Session>(s->session);
            return f(model, sess);
        },
        s->owner->model);
}

template <typename F> auto with_engine(BatchHolder *b, F &&f) {
    return std::visit([&](auto &e) { return f(*e); }, b->engine);
}

int model_device(ModelHolder *m) {
    return with_model(m, [](auto &md) { return md.device(); });
}

void set_device(ModelHolder *m) { OPWORKS_CUDA_CHECK(cudaSetDevice(model_device(m))); }

ModelHolder *load_model(const char *pack_path, unsigned sets, int max_positions) {
    if (!pack_path)
        throw std::invalid_argument("null pack path");
    opworks::PackReader probe(pack_path);
    if (probe.dtype() == "float32")
        return new ModelHolder{opworks::LlamaModel::load(pack_path, sets, max_positions)};
    if (probe.dtype() == "bfloat16")
        return new ModelHolder{opworks::LlamaModelBF16::load(pack_path, sets, max_positions)};
    throw std::runtime_error("unsupported pack dtype " + probe.dtype());
}

} // namespace

extern "C" {

void *opw_llama_load(const char *pack_path, char *err, int err_len) {
    return guard_ptr([&]() -> void * { return load_model(pack_path, 0, 8192); }, err, err_len);
}

void *opw_llama_load_ex(const char *pack_path, unsigned weight_sets, int max_positions, char *err, int err_len) {
    return guard_ptr(
        [&]() -> void * {
            if (max_positions <= 0)
                throw std::invalid_argument("max_positions must be positive");
            return load_model(pack_path, weight_sets, max_positions);
        },
        err, err_len);
}

void opw_llama_free(void *model) {
    auto *m = static_cast<ModelHolder *>(model);
    if (m) {
        cudaSetDevice(model_device(m));
        delete m;
    }
}

void *opw_llama_create_session(void *model, int max_seq_len, char *err, int err_len) {
    if (!model) {
        capture_error("null model", err, err_len);
        return nullptr;
    }
    return guard_ptr(
        [&]() -> void * {
            auto *m = static_cast<ModelHolder *>(model);
            set_device(m);
            return std::visit(
                [&](auto &md) -> void * {
                    return new SessionHolder{m, md.create_session(max_seq_len)};
                },
                m->model);
        },
        err, err_len);
}

void opw_llama_destroy_session(void *session) {
    auto *s = static_cast<SessionHolder *>(session);
    if (s) {
        cudaSetDevice(model_device(s->owner));
        delete s;
    }
}

int opw_llama_reset_session(void *session, char *err, int err_len) {
    return guard(
        [&] {
            if (!session)
                throw std::invalid_argument("null session");
            auto *s = static_cast<SessionHolder *>(session);
            set_device(s->owner);
            with_session(s, [](auto &, auto &sess) {
                sess.cache.reset();
                return 0;
            });
            return 0;
        },
        err, err_len);
}

int opw_llama_prefill(void *session, const int32_t *tokens, int n, char *err, int err_len) {
    return guard(
        [&] {
            if (!session)
                throw std::invalid_argument("null session");
            auto *s = static_cast<SessionHolder *>(session);
            if (!tokens && n > 0)
                throw std::invalid_argument("null token buffer");
            if (n < 0)
                throw std::invalid_argument("negative token count");
            set_device(s->owner);
            std::vector<int32_t> ids(tokens, tokens + static_cast<size_t>(n));
            return static_cast<int>(with_session(s, [&](auto &m, auto &sess) { return m.prefill(sess, ids); }));
        },
        err, err_len);
}

int opw_llama_decode_step(void *session, int32_t prev_token, char *err, int err_len) {
    return guard(
        [&] {
            if (!session)
                throw std::invalid_argument("null session");
            auto *s = static_cast<SessionHolder *>(session);
            set_device(s->owner);
            return static_cast<int>(
                with_session(s, [&](auto &m, auto &sess) { return m.decode_step(sess, prev_token); }));
        },
        err, err_len);
}

int opw_llama_is_eos(void *session, int32_t token, char *err, int err_len) {
    return guard(
        [&] {
            if (!session)
                throw std::invalid_argument("null session");
            auto *s = static_cast<SessionHolder *>(session);
            return with_model(s->owner, [&](auto &m) { return m.is_eos(token) ? 1 : 0; });
        },
        err, err_len);
}

int opw_llama_last_logits(void *session, float *out, int n, char *err, int err_len) {
    return guard(
        [&] {
            if (!session)
                throw std::invalid_argument("null session");
            if (!out)
                throw std::invalid_argument("null logits buffer");
            auto *s = static_cast<SessionHolder *>(session);
            set_device(s->owner);
            with_session(s, [&](auto &m, auto &sess) {
                m.copy_last_logits(sess, out, n);
                return 0;
            });
            return 0;
        },
        err, err_len);
}

int opw_llama_vocab_size(void *session) {
    auto *s = static_cast<SessionHolder *>(session);
    return with_model(s->owner, [](auto &m) { return m.config().vocab_size; });
}

const char *opw_llama_last_error(void) { return g_last_error.c_str(); }

int opw_llama_set_device(int device) {
    return guard(
        [&] {
            int count = 0;
            OPWORKS_CUDA_CHECK(cudaGetDeviceCount(&count));
            if (device < 0 || device >= count)
                throw std::invalid_argument("device index out of range");
            OPWORKS_CUDA_CHECK(cudaSetDevice(device));
            return 0;
        },
        nullptr, 0);
}

int opw_llama_model_info(void *model, int32_t *out8, char *err, int err_len) {
    return guard(
        [&] {
            if (!model || !out8)
                throw std::invalid_argument("null argument");
            auto *m = static_cast<ModelHolder *>(model);
            with_model(m, [&](auto &md) {
                const auto &c = md.config();
                out8[0] = c.num_layers;
                out8[1] = c.hidden_size;
                out8[2] = c.intermediate_size;
                out8[3] = c.num_q_heads;
                out8[4] = c.num_kv_heads;
                out8[5] = c.head_dim;
                out8[6] = c.vocab_size;
                out8[7] = md.device();
                return 0;
            });
            return 0;
        },
        err, err_len);
}

void *opw_llama_create_batch(void *model, int max_batch, int max_seq_len, int precision, int prefill_rows, char *err,
                             int err_len) {
    return guard_ptr(
        [&]() -> void * {
            if (!model)
                throw std::invalid_argument("null model");
            if (precision != 0 && precision != 1)
                throw std::invalid_argument("precision must be 0 (accurate) or 1 (fast)");
            auto *m = static_cast<ModelHolder *>(model);
            set_device(m);
            auto *b = new BatchHolder{m, {}};
            try {
                std::visit(
                    [&](auto &md) {
                        b->engine = md.create_engine(max_batch, max_seq_len, static_cast<opworks::Precision>(precision),
                                                     prefill_rows);
                    },
                    m->model);
            } catch (...) {
                delete b;
                throw;
            }
            return b;
        },
        err, err_len);
}

int opw_llama_nccl_unique_id(char *out, char *err, int err_len) {
    return guard(
        [&] {
            if (!out)
                throw std::invalid_argument("null output");
            opworks::NcclLite::get().unique_id(out);
            return 0;
        },
        err, err_len);
}

void *opw_llama_create_batch_tp(void *model, int max_batch, int max_seq_len, int prefill_rows, int tp_rank,
                                int tp_world, const char *nccl_id, char *err, int err_len) {
    return guard_ptr(
        [&]() -> void * {
            if (!model || !nccl_id)
                throw std::invalid_argument("null model or NCCL id");
            auto *m = static_cast<ModelHolder *>(model);
            set_device(m);
            auto *b = new BatchHolder{m, {}};
            try {
                opworks::TensorParallel tp;
                tp.rank = tp_rank;
                tp.world = tp_world;
                tp.nccl_id = nccl_id;
                std::visit(
                    [&](auto &md) {
                        b->engine = md.create_engine(max_batch, max_seq_len, opworks::Precision::kFast, prefill_rows,
                                                     tp);
                    },
                    m->model);
            } catch (...) {
                delete b;
                throw;
            }
            return b;
        },
        err, err_len);
}

int opw_llama_batch_tp_ipc_handle(void *batch, char *out128, char *err, int err_len) {
    return guard(
        [&] {
            if (!batch || !out128)
                throw std::invalid_argument("null batch or output");
            auto *b = static_cast<BatchHolder *>(batch);
            set_device(b->owner);
            return with_engine(b, [&](auto &e) {
                e.tp_ipc_handles(out128);
                return 0;
            });
        },
        err, err_len);
}

int opw_llama_batch_tp_open_peers(void *batch, const char *handles, char *err, int err_len) {
    return guard(
        [&] {
            if (!batch || !handles)
                throw std::invalid_argument("null batch or handles");
            auto *b = static_cast<BatchHolder *>(batch);
            set_device(b->owner);
            return with_engine(b, [&](auto &e) {
                e.tp_open_peers(handles);
                return 0;
            });
        },
        err, err_len);
}

void opw_llama_destroy_batch(void *batch) {
    auto *b = static_cast<BatchHolder *>(batch);
    if (b) {
        cudaSetDevice(model_device(b->owner));
        delete b;
    }
}

int opw_llama_batch_reset(void *batch, int slot, char *err, int err_len) {
    return guard(
        [&] {
            if (!batch)
                throw std::invalid_argument("null batch");
            auto *b = static_cast<BatchHolder *>(batch);
            set_device(b->owner);
            with_engine(b, [&](auto &e) {
                e.reset(slot);
                return 0;
            });
            return 0;
        },
        err, err_len);
}

int opw_llama_batch_length(void *batch, int slot) {
    if (!batch)
        return -1;
    auto *b = static_cast<BatchHolder *>(batch);
    try {
        return with_engine(b, [&](auto &e) { return e.length(slot); });
    } catch (...) {
        return -1;
    }
}

int opw_llama_batch_prefill(void *batch, int slot, const int32_t *tokens, int n, float temperature, float top_p,
                            double uniform, uint64_t seed, char *err, int err_len) {
    return guard(
        [&] {
            if (!batch)
                throw std::invalid_argument("null batch");
            if (!tokens && n > 0)
                throw std::invalid_argument("null token buffer");
            auto *b = static_cast<BatchHolder *>(batch);
            set_device(b->owner);
            opworks::SampleArgs sa;
            sa.temperature = temperature;
            sa.top_p = top_p;
            sa.uniform = uniform;
            sa.seed = seed;
            sa.step = 0;
            return static_cast<int>(with_engine(b, [&](auto &e) { return e.prefill(slot, tokens, n, sa); }));
        },
        err, err_len);
}

int opw_llama_batch_decode(void *batch, int n, const int32_t *slots, const int32_t *prev_tokens,
                           const float *temperature, const float *top_p, const double *uniforms,
                           const uint64_t *seeds, const int32_t *steps, int32_t *out_tokens, char *err, int err_len) {
    return guard(
        [&] {
            if (!batch)
                throw std::invalid_argument("null batch");
            if (n <= 0 || !slots || !prev_tokens || !out_tokens)
                throw std::invalid_argument("decode needs n > 0, slots, prev_tokens and out_tokens");
            auto *b = static_cast<BatchHolder *>(batch);
            set_device(b->owner);
            std::vector<opworks::SampleArgs> sa(static_cast<size_t>(n));
            for (int i = 0; i < n; ++i) {
                sa[i].temperature = temperature ? temperature[i] : 0.f;
                sa[i].top_p = top_p ? top_p[i] : 1.f;
                sa[i].uniform = uniforms ? uniforms[i] : -1.0;
                sa[i].seed = seeds ? seeds[i] : 0;
                sa[i].step = steps ? steps[i] : 0;
            }
            with_engine(b, [&](auto &e) {
                e.decode(n, slots, prev_tokens, sa.data(), out_tokens);
                return 0;
            });
            return 0;
        },
        err, err_len);
}

int opw_llama_batch_decode_multi(void *batch, int n, const int32_t *slots, const int32_t *prev_tokens,
                                 const float *temperature, const float *top_p, const double *uniforms,
                                 const uint64_t *seeds, const int32_t *steps0, int steps, int eos_id,
                                 int32_t *out_tokens, int32_t *out_counts, char *err, int err_len) {
    return guard(
        [&] {
            if (!batch)
                throw std::invalid_argument("null batch");
            if (n <= 0 || steps <= 0 || !slots || !prev_tokens || !out_tokens || !out_counts)
                throw std::invalid_argument("multi-step decode needs n > 0, steps > 0, slots, prev_tokens and outputs");
            auto *b = static_cast<BatchHolder *>(batch);
            set_device(b->owner);
            std::vector<opworks::SampleArgs> sa(static_cast<size_t>(n));
            for (int i = 0; i < n; ++i) {
                sa[i].temperature = temperature ? temperature[i] : 0.f;
                sa[i].top_p = top_p ? top_p[i] : 1.f;
                sa[i].uniform = uniforms ? uniforms[i] : -1.0;
                sa[i].seed = seeds ? seeds[i] : 0;
                sa[i].step = steps0 ? steps0[i] : 0;
            }
            with_engine(b, [&](auto &e) {
                e.decode_multi(n, slots, prev_tokens, sa.data(), steps, uniforms, eos_id, out_tokens, out_counts);
                return 0;
            });
            return 0;
        },
        err, err_len);
}

int opw_llama_batch_logits(void *batch, int row, float *out, int n, char *err, int err_len) {
    return guard(
        [&] {
            if (!batch || !out)
                throw std::invalid_argument("null argument");
            auto *b = static_cast<BatchHolder *>(batch);
            set_device(b->owner);
            with_engine(b, [&](auto &e) {
                e.copy_logits(row, out, n);
                return 0;
            });
            return 0;
        },
        err, err_len);
}

void *opw_llama_batch_stream(void *batch) {
    if (!batch)
        return nullptr;
    auto *b = static_cast<BatchHolder *>(batch);
    return with_engine(b, [](auto &e) { return static_cast<void *>(e.stream()); });
}

int opw_llama_batch_io_bytes(void *batch, int n, int64_t *out2) {
    if (!batch || !out2)
        return -1;
    auto *b = static_cast<BatchHolder *>(batch);
    with_engine(b, [&](auto &e) {
        out2[0] = e.decode_h2d_bytes();
        out2[1] = e.decode_d2h_bytes(n);
        return 0;
    });
    return 0;
}

int opw_llama_batch_profile(void *batch, int n, int iters, float *ms_per_step, int32_t *launches_per_step,
                            char *labels, int max_kernels, char *err, int err_len) {
    return guard(
        [&] {
            if (!batch || !ms_per_step || !launches_per_step || !labels)
                throw std::invalid_argument("null argument");
            auto *b = static_cast<BatchHolder *>(batch);
            set_device(b->owner);
            return with_engine(b, [&](auto &e) {
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
        },
        err, err_len);
}

} // extern "C"
