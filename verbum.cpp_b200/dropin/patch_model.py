"""Writes the engine-backed verbum::Model: the reference's model.h and
model.cpp with their CUDA half re-pointed at libverbum_b200.so.

    python patch_model.py REF_ROOT OUT_DIR

Reads REF_ROOT/core/include/verbum/model.h and REF_ROOT/core/src/model.cpp
where they lie and writes patched copies to OUT_DIR/include/verbum/model.h and
OUT_DIR/src/model.cpp (a build directory, never committed).  The edits are the
ones a maintainer would make (compiled in under VERBUM_B200, next to the
reference's own code, which stays in the #else branches):

  model.h   -- includes verbum_b200.h; Model gains the engine handle, a
               destructor that releases it, and no copies (one engine each);
  model.cpp -- to_cuda() (model.cpp:367-443) creates the engine and uploads
               the weights: f32 tensors, or -- after quantize() -- the
               reference's own QuantLayer int8 rows and scales (the
               reference refuses quantized + CUDA, model.cpp:374-377);
               step_cuda() (446-497) is one vb_engine_step; reset_cache()
               (277-282) also resets the engine's cache once it exists.

Each edit is anchored on a declaration or signature that must occur exactly
once; a reference that no longer matches stops the build with the anchor's
name rather than producing a half-patched file.
"""
import re
import sys
from pathlib import Path


def once(text, pattern, what):
    m = list(re.finditer(pattern, text, flags=re.M))
    if len(m) != 1:
        raise SystemExit(f"patch_model: anchor '{what}' found {len(m)} times (expected 1)")
    return m[0]


def body_span(text, header_match, what):
    """(start, end) of the {...} body that follows a function header."""
    i = text.index("{", header_match.end() - 1)
    depth = 0
    for j in range(i, len(text)):
        if text[j] == "{":
            depth += 1
        elif text[j] == "}":
            depth -= 1
            if depth == 0:
                return i, j
    raise SystemExit(f"patch_model: unbalanced body of '{what}'")


def wrap_body(text, sig_pattern, what, engine_body):
    m = once(text, sig_pattern, what)
    a, b = body_span(text, m, what)
    original = text[a + 1:b]
    new = "{\n#ifdef VERBUM_B200\n" + engine_body + "#else" + original + "#endif\n}"
    return text[:a] + new + text[b + 1:]


TO_CUDA = r"""
    if (cuda_) return;
    if (vb_device_count() == 0) throw std::runtime_error("no CUDA device found");
    if (caches_.empty()) throw std::runtime_error("call reset_cache() before to_cuda()");
    vb_config c{};
    c.hidden = cfg_.hidden_size;
    c.layers = cfg_.num_hidden_layers;
    c.heads = cfg_.num_attention_heads;
    c.kv_heads = cfg_.num_key_value_heads;
    c.head_dim = cfg_.head_dim;
    c.ffn = cfg_.intermediate_size;
    c.vocab = cfg_.vocab_size;
    c.rope_positions = cfg_.max_position_embeddings > 4096 ? 4096 : cfg_.max_position_embeddings;
    c.eps = cfg_.rms_norm_eps;
    c.theta = cfg_.rope_theta;
    vb_b200_check(vb_engine_create(&c, /*device=*/0, &vb_));
    vb_b200_check(vb_engine_set_globals(vb_, lm_head_vec().data(), final_norm_.data()));
    for (int i = 0; i < cfg_.num_hidden_layers; i++) {
        const LayerWeights& L = layers_[i];
        if (quantized_) {
            const QuantLayer& Q = qlayers_[i];
            vb_layer_host_q8 h{};
            h.input_norm = L.input_norm.data();
            h.post_norm = L.post_attention_norm.data();
            h.q_norm = L.attn.q_norm.data();
            h.k_norm = L.attn.k_norm.data();
            h.wq = Q.q_proj.data.data(); h.sq = Q.q_proj.scales.data();
            h.wk = Q.k_proj.data.data(); h.sk = Q.k_proj.scales.data();
            h.wv = Q.v_proj.data.data(); h.sv = Q.v_proj.scales.data();
            h.wo = Q.o_proj.data.data(); h.so = Q.o_proj.scales.data();
            h.wg = Q.gate_proj.data.data(); h.sg = Q.gate_proj.scales.data();
            h.wu = Q.up_proj.data.data(); h.su = Q.up_proj.scales.data();
            h.wd = Q.down_proj.data.data(); h.sd = Q.down_proj.scales.data();
            vb_b200_check(vb_engine_set_layer_q8(vb_, i, &h));
        } else {
            vb_layer_host h{};
            h.input_norm = L.input_norm.data();
            h.post_norm = L.post_attention_norm.data();
            h.wq = L.attn.q_proj.data();
            h.wk = L.attn.k_proj.data();
            h.wv = L.attn.v_proj.data();
            h.wo = L.attn.o_proj.data();
            h.q_norm = L.attn.q_norm.data();
            h.k_norm = L.attn.k_norm.data();
            h.wg = L.ffn.gate_proj.data();
            h.wu = L.ffn.up_proj.data();
            h.wd = L.ffn.down_proj.data();
            vb_b200_check(vb_engine_set_layer(vb_, i, &h));
        }
    }
    vb_b200_check(vb_engine_reset_cache(vb_, caches_[0].max_seq));
    cuda_ = true;
"""

STEP_CUDA = r"""
    if (caches_.empty()) throw std::runtime_error("call reset_cache() first");
    vb_b200_check(vb_engine_step(vb_, token_id, logits.data()));
    for (auto& c : caches_) c.len++;
"""

HELPERS = r"""
#ifdef VERBUM_B200
namespace {
void vb_b200_check(vb_status s) {
    if (s != VB_OK) throw std::runtime_error(vb_last_error());
}
}  // namespace
#endif
"""

DTOR = r"""
#ifdef VERBUM_B200
Model::~Model() {
    if (vb_) vb_engine_destroy(vb_);
}
#endif
"""


def patch_header(h):
    m = once(h, r'^#include "verbum/cuda_backend.h"\s*$', "model.h: #include cuda_backend.h")
    h = h[:m.end()] + '\n#ifdef VERBUM_B200\n#include "verbum_b200.h"\n#endif' + h[m.end():]
    m = once(h, r"^\s*bool cuda_ = false;\s*$", "model.h: bool cuda_ member")
    h = h[:m.end()] + ("\n#ifdef VERBUM_B200\n    vb_engine* vb_ = nullptr;\n\npublic:\n    ~Model();\n"
                       "    Model(const Model&) = delete;\n    Model& operator=(const Model&) = delete;\n\n"
                       "private:\n#endif") + h[m.end():]
    return h


def patch_source(s):
    last_inc = list(re.finditer(r"^#include .*$", s, flags=re.M))
    if not last_inc:
        raise SystemExit("patch_model: no #include in model.cpp")
    k = last_inc[-1].end()
    s = s[:k] + "\n" + s[k:]
    ns = once(s, r"^namespace verbum \{\s*$", "model.cpp: namespace verbum")
    s = s[:ns.end()] + "\n" + HELPERS + s[ns.end():]
    s = wrap_body(s, r"^void Model::to_cuda\(\)\s*\{", "Model::to_cuda", TO_CUDA)
    s = wrap_body(s, r"^void Model::step_cuda\(int token_id, Tensor& logits\)\s*\{", "Model::step_cuda",
                  STEP_CUDA)
    m = once(s, r"^void Model::reset_cache\(int max_seq\)\s*\{", "Model::reset_cache")
    a, b = body_span(s, m, "Model::reset_cache")
    s = s[:b] + "#ifdef VERBUM_B200\n    if (vb_) vb_b200_check(vb_engine_reset_cache(vb_, max_seq));\n#endif\n" + s[b:]
    end = once(s, r"^\}\s*//\s*namespace verbum\s*$", "model.cpp: end of namespace verbum")
    s = s[:end.start()] + DTOR + "\n" + s[end.start():]
    return s


def main():
    ref, out = Path(sys.argv[1]), Path(sys.argv[2])
    h = (ref / "core" / "include" / "verbum" / "model.h").read_text()
    s = (ref / "core" / "src" / "model.cpp").read_text()
    (out / "include" / "verbum").mkdir(parents=True, exist_ok=True)
    (out / "src").mkdir(parents=True, exist_ok=True)
    (out / "include" / "verbum" / "model.h").write_text(patch_header(h))
    (out / "src" / "model.cpp").write_text(patch_source(s))


if __name__ == "__main__":
    main()
