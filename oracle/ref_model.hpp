// ref_model.hpp -- TEST INFRASTRUCTURE ONLY: builds a parakeet::ParakeetCtcModel
// (the reference's model type, src/parakeet_ctc.h) from a pk_model_desc, with every
// tensor in host memory as a ggml_tensor of the host-only ggml stand-in
// (oracle/ggml_host/). Shared by the checker around the reference's own decoder
// (ref_decoder_shim.cpp) and the harness that drives the C++ drop-in shim
// (tests/shim/shim_harness.cpp) through the same model.
#pragma once

#include "parakeet_ctc.h"

#include "ggml.h"

#include "parakeet_cuda.h"

#include <algorithm>
#include <memory>
#include <string>
#include <vector>

namespace refmodel {

struct Blob {
    ggml_tensor t{};
    std::vector<uint8_t> bytes;
};

struct Model {
    parakeet::ParakeetCtcModel model;
    std::vector<std::unique_ptr<Blob>> blobs;
    bool is_tdt = true;
    int max_symbols = 10;

    ggml_tensor * tensor(const pk_tensor & src) {
        if (!src.data) return nullptr;
        auto b = std::make_unique<Blob>();
        b->bytes.assign(static_cast<const uint8_t *>(src.data), static_cast<const uint8_t *>(src.data) + src.nbytes);
        ggml_tensor & t = b->t;
        t.type = (ggml_type) src.type;
        t.ne[0] = src.ne0;
        t.ne[1] = src.ne1 > 0 ? src.ne1 : 1;
        t.ne[2] = t.ne[3] = 1;
        const ggml_type_traits * tr = ggml_get_type_traits(t.type);
        t.nb[0] = tr ? tr->type_size : 0;
        t.nb[1] = tr ? (size_t) (t.ne[0] / tr->blck_size) * tr->type_size : 0;
        t.nb[2] = t.nb[1] * (size_t) t.ne[1];
        t.nb[3] = t.nb[2];
        t.data = b->bytes.data();
        blobs.push_back(std::move(b));
        return &blobs.back()->t;
    }

    // Fills `model` from the descriptor (hyper-parameters as the GGUF loader sets
    // them, src/parakeet_ctc.cpp:424-460; tokenizer pieces shaped "<...>" where the
    // descriptor flags a special piece).
    void fill(const pk_model_desc & d) {
        parakeet::ParakeetCtcModel & M = model;
        is_tdt = d.model_type == PK_MODEL_TDT;
        M.model_type = is_tdt ? parakeet::ParakeetModelType::TDT : parakeet::ParakeetModelType::EOU;
        M.encoder_cfg.d_model = d.d_enc;
        M.vocab_size = d.vocab_size;
        M.blank_id = d.blank_id;
        M.eou_id = d.eou_id;
        M.eob_id = d.eob_id;
        M.vocab.pieces.resize((size_t) std::max(0, d.n_vocab_pieces));
        for (int32_t i = 0; i < d.n_vocab_pieces; ++i)
            M.vocab.pieces[(size_t) i] = (d.special_piece && d.special_piece[i]) ? "<s" + std::to_string(i) + ">"
                                                                             : "p" + std::to_string(i);
        M.vocab.blank_id = d.blank_id;
        std::vector<parakeet::TdtLstmLayer> lstm((size_t) std::max(0, d.n_layers));
        for (int32_t l = 0; l < d.n_layers; ++l) {
            lstm[(size_t) l].w_ih = tensor(d.lstm[l].w_ih);
            lstm[(size_t) l].w_hh = tensor(d.lstm[l].w_hh);
            lstm[(size_t) l].b_ih = tensor(d.lstm[l].b_ih);
            lstm[(size_t) l].b_hh = tensor(d.lstm[l].b_hh);
        }
        max_symbols = d.max_symbols_per_step;
        if (is_tdt) {
            M.encoder_cfg.tdt_pred_hidden = d.pred_hidden;
            M.encoder_cfg.tdt_joint_hidden = d.joint_hidden;
            M.encoder_cfg.tdt_pred_rnn_layers = d.n_layers;
            M.encoder_cfg.tdt_num_durations = d.num_durations;
            M.tdt_durations.assign(d.durations, d.durations + d.num_durations);
            set_weights(M.tdt, d, lstm);
        } else {
            M.encoder_cfg.eou_pred_hidden = d.pred_hidden;
            M.encoder_cfg.eou_joint_hidden = d.joint_hidden;
            M.encoder_cfg.eou_pred_rnn_layers = d.n_layers;
            M.encoder_cfg.eou_max_symbols_per_step = d.max_symbols_per_step;
            set_weights(M.eou, d, lstm);
        }
    }

    template <class W>
    void set_weights(W & w, const pk_model_desc & d, const std::vector<parakeet::TdtLstmLayer> & lstm) {
        w.predict_embed = tensor(d.embed);
        w.lstm = lstm;
        w.joint_enc_w = tensor(d.joint_enc_w);
        w.joint_enc_b = tensor(d.joint_enc_b);
        w.joint_pred_w = tensor(d.joint_pred_w);
        w.joint_pred_b = tensor(d.joint_pred_b);
        w.joint_out_w = tensor(d.joint_out_w);
        w.joint_out_b = tensor(d.joint_out_b);
    }
};

}  // namespace refmodel
