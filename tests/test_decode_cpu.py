"""The decode harness (xdna.cpp_b200/decode_harness.py) on a tiny
Qwen2-style config, on the CPU: driven once by the oracle's Q4_0 matmul and
once by a float64 product of the gguf-dequantised weights (a second,
independent implementation), it must produce the same greedy tokens, with
per-step logits that agree closely.  This checks the harness's host
arithmetic (RMSNorm, RoPE, grouped-query attention, SwiGLU) and its greedy
loop; the GPU test drives the same harness with the plugin."""
from __future__ import annotations

import numpy as np

from helpers import normal_weights

TINY = dict(hidden=256, layers=2, heads=4, kv_heads=2, head_dim=64, inter=512, vocab=1000, theta=1.0e6, eps=1.0e-6)


def test_harness_greedy_decode_two_matmul_paths_agree(O):
    import gguf
    from gguf.quants import dequantize

    import decode_harness as D

    shapes = D.mat_shapes(TINY)
    raws, deq = {}, {}
    for i, (layer, name) in enumerate(D.weight_keys(TINY)):
        N, K = shapes[name]
        raws[(layer, name)] = O.quantize(O.Q4_0, normal_weights(N, K, seed=500 + i), nthreads=4)
        deq[(layer, name)] = dequantize(raws[(layer, name)].reshape(N, -1), gguf.GGMLQuantizationType.Q4_0).astype(
            np.float64).reshape(N, K)

    def mm_oracle(keys, x):
        return [O.gemv(O.Q4_0, raws[k], shapes[k[1]][0], shapes[k[1]][1], np.ascontiguousarray(x), nthreads=4)
                for k in keys]

    def mm_f64(keys, x):
        return [(deq[k] @ x.astype(np.float64)).astype(np.float32) for k in keys]

    prompt = D.prompt_ids(TINY, 5, 6)
    t1, l1 = D.Decoder(TINY, 5, mm_oracle).generate(prompt, 10)
    t2, l2 = D.Decoder(TINY, 5, mm_f64).generate(prompt, 10)
    assert t1 == t2
    for a, b in zip(l1, l2):
        cos = float(a.astype(np.float64) @ b / (np.linalg.norm(a) * np.linalg.norm(b)))
        assert cos >= 0.99999, cos


def test_harness_matches_transformers_qwen2(O):
    """The harness's host arithmetic is Qwen2's: transformers' Qwen2ForCausalLM
    with the same weights (the dequantised Q4_0 matrices, the harness's
    embedding rows, zero q/k/v biases, unit norms) gives the same greedy
    tokens and close logits for the tiny config."""
    torch = __import__("torch")
    transformers = __import__("transformers")
    import gguf
    from gguf.quants import dequantize

    import decode_harness as D

    seed = 6
    shapes = D.mat_shapes(TINY)
    deq = {}
    for i, (layer, name) in enumerate(D.weight_keys(TINY)):
        N, K = shapes[name]
        raw = O.quantize(O.Q4_0, normal_weights(N, K, seed=700 + i), nthreads=4)
        deq[(layer, name)] = dequantize(raw.reshape(N, -1), gguf.GGMLQuantizationType.Q4_0).astype(
            np.float32).reshape(N, K)

    def mm_f64(keys, x):
        return [(deq[k].astype(np.float64) @ x.astype(np.float64)).astype(np.float32) for k in keys]

    prompt = D.prompt_ids(TINY, seed, 5)
    toks, logits = D.Decoder(TINY, seed, mm_f64).generate(prompt, 8)

    cfg = transformers.Qwen2Config(hidden_size=TINY["hidden"], intermediate_size=TINY["inter"],
                                   num_hidden_layers=TINY["layers"], num_attention_heads=TINY["heads"],
                                   num_key_value_heads=TINY["kv_heads"], vocab_size=TINY["vocab"],
                                   rms_norm_eps=TINY["eps"], rope_theta=TINY["theta"], tie_word_embeddings=False,
                                   max_position_embeddings=64)
    model = transformers.Qwen2ForCausalLM(cfg).eval()
    with torch.no_grad():
        model.model.embed_tokens.weight.copy_(torch.from_numpy(
            np.stack([D.embedding_row(TINY, seed, t) for t in range(TINY["vocab"])])))
        proj = {"q": "self_attn.q_proj", "k": "self_attn.k_proj", "v": "self_attn.v_proj", "o": "self_attn.o_proj",
                "gate": "mlp.gate_proj", "up": "mlp.up_proj", "down": "mlp.down_proj"}
        for layer in range(TINY["layers"]):
            blk = model.model.layers[layer]
            for name, path in proj.items():
                lin = blk.get_submodule(path)
                lin.weight.copy_(torch.from_numpy(deq[(layer, name)]))
                if lin.bias is not None:
                    lin.bias.zero_()
            blk.input_layernorm.weight.fill_(1.0)
            blk.post_attention_layernorm.weight.fill_(1.0)
        model.model.norm.weight.fill_(1.0)
        model.lm_head.weight.copy_(torch.from_numpy(deq[(TINY["layers"], "lm_head")]))
        out = model.generate(torch.tensor([prompt]), max_new_tokens=8, do_sample=False, output_scores=True,
                             return_dict_in_generate=True, pad_token_id=0)
    ref = out.sequences[0, len(prompt):].tolist()
    assert toks == ref, (toks, ref)
    for a, b in zip(logits, out.scores):
        b = b[0].double().numpy()
        cos = float(a.astype(np.float64) @ b / (np.linalg.norm(a) * np.linalg.norm(b)))
        assert cos >= 0.9999, cos
