"""The oracle's whole forward against an independent implementation:
transformers' Qwen2 model, built from the GGUF's configuration (nothing
downloaded), run in float64 over the oracle's own dequantized weights.  It
checks the semantics the oracle restates (half-split RoPE at theta, GQA
attention, RMSNorm, SwiGLU, q/k/v biases, untied output) and bounds the
oracle's f32 error.  CPU only."""

import numpy as np
import pytest

from furnace_b200 import synth

torch = pytest.importorskip("torch")
pytest.importorskip("transformers")


def _hf_model(orc, ref):
    from transformers import Qwen2Config, Qwen2ForCausalLM

    tied = True
    try:
        ref.tensor("output.weight")
        tied = False
    except Exception:
        pass
    cfg = Qwen2Config(vocab_size=ref.vocab, hidden_size=ref.hidden, intermediate_size=ref.ffn,
                      num_hidden_layers=ref.n_layers, num_attention_heads=ref.n_heads,
                      num_key_value_heads=ref.n_kv_heads, max_position_embeddings=ref.context_length,
                      rms_norm_eps=ref.rms_eps, tie_word_embeddings=tied,
                      rope_parameters={"rope_type": "default", "rope_theta": ref.rope_theta})
    cfg._attn_implementation = "eager"
    model = Qwen2ForCausalLM(cfg).double().eval()

    def w(name):  # GGUF dims are (in, out): a row-major [out, in] matrix
        dt, dims, raw = ref.tensor(name)
        vals = orc.dequantize(dt, raw, int(np.prod(dims)))
        return torch.from_numpy(vals.astype(np.float64).reshape(list(reversed(dims))))

    sd = {"model.embed_tokens.weight": w("token_embd.weight"), "model.norm.weight": w("output_norm.weight")}
    if not tied:
        sd["lm_head.weight"] = w("output.weight")
    for i in range(ref.n_layers):
        p, q = f"blk.{i}.", f"model.layers.{i}."
        for a, b in (("attn_q", "self_attn.q_proj"), ("attn_k", "self_attn.k_proj"), ("attn_v", "self_attn.v_proj")):
            sd[q + b + ".weight"] = w(p + a + ".weight")
            sd[q + b + ".bias"] = w(p + a + ".bias")
        sd[q + "self_attn.o_proj.weight"] = w(p + "attn_output.weight")
        sd[q + "mlp.gate_proj.weight"] = w(p + "ffn_gate.weight")
        sd[q + "mlp.up_proj.weight"] = w(p + "ffn_up.weight")
        sd[q + "mlp.down_proj.weight"] = w(p + "ffn_down.weight")
        sd[q + "input_layernorm.weight"] = w(p + "attn_norm.weight")
        sd[q + "post_attention_layernorm.weight"] = w(p + "ffn_norm.weight")
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected and all(k == "lm_head.weight" for k in missing), (missing, unexpected)
    return model


@pytest.mark.parametrize("over", [{}, {"hidden": 1792, "n_heads": 14, "n_kv_heads": 2, "n_layers": 2},
                                  {"tied": True, "n_layers": 2}],
                         ids=["tiny-hd64", "hd128-g7", "tied"])
def test_oracle_forward_matches_float64_transformers(orc, tmp_path, over):
    from oracle import oracle

    path = synth.write(synth.spec("tiny", **over), str(tmp_path / "m.gguf"))
    ref = oracle.Model(path)
    hf = _hf_model(orc, ref)
    ids = [int(x) for x in synth.prompt_ids(ref.vocab, 24, seed=3)]
    with torch.no_grad():
        want = hf(torch.tensor([ids])).logits[0].numpy()  # [T, vocab], float64
    # every position through forward_cached one token at a time, then the
    # last position of a batched call
    kv = ref.kv_new(64)
    scale = np.abs(want).max()
    for t, tok in enumerate(ids):
        got = ref.forward_cached([tok], kv)
        assert np.abs(got - want[t]).max() <= 1e-5 * max(1.0, scale), t
    got = ref.forward_last(ids)
    assert np.abs(got - want[-1]).max() <= 1e-5 * max(1.0, scale)
    # greedy continuation: identical ids unless two logits are within the
    # f32 error (checked on the float64 logits)
    seq = list(ids)
    kv2 = ref.kv_new(64)
    lg = ref.forward_cached(seq, kv2)
    for _ in range(12):
        nxt = int(np.argmax(lg))
        with torch.no_grad():
            h = hf(torch.tensor([seq])).logits[0, -1].numpy()
        top2 = np.sort(h)[-2:]
        if top2[1] - top2[0] > 1e-4:
            assert nxt == int(np.argmax(h))
        seq.append(nxt)
        lg = ref.forward_cached([nxt], kv2)
