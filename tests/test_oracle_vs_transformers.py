"""The oracle's whole MoE block against Hugging Face transformers' implementations
of the same models, run in float64 on the CPU.

The reference (rs-gallium) cannot run here: it is Rust, and its arithmetic
lives in candle, which is not vendored.  No reference test pins its router,
activation, GEMMs or combine.  transformers (installed in this image) carries
an independent implementation of each model's MoE block:

* GPT-OSS: ``GptOssMLP`` (router ``F.linear`` + top-k + softmax over the k
  logits, clamped SwiGLU with alpha 1.702 and limit 7, per-expert biases,
  routing-weighted ``index_add_``) and the safetensors MXFP4 unpacking
  ``convert_moe_packed_tensors`` (low nibble -> even element, high -> odd,
  ``ldexp`` by scale - 127).  The reference follows the same layout
  (crates/gallium-models/src/gpt_oss.rs:145-164, 166-231).
* LFM2.5: ``Lfm2MoeSparseMoeBlock`` (sigmoid router, selection by sigmoid +
  expert bias, weights renormalised over the top k, SiLU-gated experts
  without biases), as lfm2moe_q.rs:234-313.

The oracle computes in f32 in the reference's order; transformers here in
float64.  Bars (written in each test): indices equal, outputs within
max-abs 1e-3 and mean-rel 1e-5 (measured: max-abs 0.8-2.2e-5, mean-rel
1.5-4.9e-7).  transformers
unpacks a zero E8M0 scale to 2^-127 times the code where the reference gives
0 (gpt_oss.rs:152), so the unpacking check uses scale bytes 1..254.
"""
import numpy as np
import pytest

import oracle
from gallium_b200 import synth

torch = pytest.importorskip("torch")
pytest.importorskip("transformers")

MAX_ABS = 1e-3
MEAN_REL = 1e-5


def _close(got, want, what, max_abs_bar=MAX_ABS, mean_rel_bar=MEAN_REL):
    err = np.abs(np.asarray(got, np.float64) - np.asarray(want, np.float64))
    max_abs = float(err.max())
    mean_rel = float(err.sum() / np.abs(want).sum())
    assert max_abs <= max_abs_bar and mean_rel <= mean_rel_bar, (what, max_abs, mean_rel)


def _f64(bits):
    return torch.from_numpy(synth.bf16_bits_to_f32(bits).astype(np.float64))


def test_safetensors_mxfp4_unpacking_matches_transformers_bit_for_bit():
    from transformers.integrations.mxfp4 import convert_moe_packed_tensors

    layer = synth.gptoss_layer(n_experts=2, hidden=256, inter=128, top_k=2, seed=4, scale_lo=1,
                               scale_hi=254)
    with np.errstate(over="ignore"):
        hf = convert_moe_packed_tensors(torch.from_numpy(layer.gu_blocks),
                                        torch.from_numpy(layer.gu_scales),
                                        dtype=torch.float32).numpy()  # [E, H, 2I]
        for e in range(2):
            ours = oracle.mxfp4_split_dequant(layer.gu_blocks[e], layer.gu_scales[e])  # [2I, H]
            assert np.array_equal(ours.T.view(np.uint32), hf[e].view(np.uint32)), e


@pytest.mark.parametrize("skewed", [False, True])
def test_gptoss_block_matches_transformers_gpt_oss_mlp(skewed):
    from transformers.integrations.mxfp4 import convert_moe_packed_tensors
    from transformers.models.gpt_oss.configuration_gpt_oss import GptOssConfig
    from transformers.models.gpt_oss.modeling_gpt_oss import GptOssMLP

    E, H, I, K, T = 8, 128, 96, 4, 24
    layer = synth.gptoss_layer(n_experts=E, hidden=H, inter=I, top_k=K, seed=3, skewed=skewed)
    cfg = GptOssConfig(hidden_size=H, intermediate_size=I, num_local_experts=E,
                       num_experts_per_tok=K, num_hidden_layers=1, num_attention_heads=4,
                       num_key_value_heads=1, head_dim=32, vocab_size=16)
    mlp = GptOssMLP(cfg).double().eval()
    gu = convert_moe_packed_tensors(torch.from_numpy(layer.gu_blocks),
                                    torch.from_numpy(layer.gu_scales), dtype=torch.float32)
    dn = convert_moe_packed_tensors(torch.from_numpy(layer.dn_blocks),
                                    torch.from_numpy(layer.dn_scales), dtype=torch.float32)
    x = synth.tokens(T, H, seed=5)
    with torch.no_grad():
        mlp.router.weight.copy_(_f64(layer.router_w))
        mlp.router.bias.copy_(_f64(layer.router_b))
        mlp.experts.gate_up_proj.copy_(gu.double())
        mlp.experts.down_proj.copy_(dn.double())
        mlp.experts.gate_up_proj_bias.copy_(_f64(layer.gu_bias))
        mlp.experts.down_proj_bias.copy_(_f64(layer.dn_bias))
        xt = torch.from_numpy(x.astype(np.float64))
        logits, scores, hf_idx = mlp.router(xt)
        hf_out, _ = mlp(xt[None])
    # selection is compared only where the k-th and (k+1)-th logits are apart
    top = torch.sort(logits, dim=-1, descending=True).values
    assert float((top[:, K - 1] - top[:, K]).min()) > 1e-6
    out, idx, w = oracle.OracleMoe(layer).forward(x)
    np.testing.assert_array_equal(idx, hf_idx.numpy())
    np.testing.assert_allclose(w, scores.numpy(), rtol=0, atol=1e-6)
    _close(out, hf_out[0].numpy(), f"GPT-OSS block, skewed={skewed}")


def test_gptoss_block_at_hidden_2880_matches_transformers():
    """The real hidden and intermediate sizes (2880), 4 experts, top-2: the
    f32 sums over K = 2880 put outputs near 1.8e3, so the absolute bar is
    1e-2 here (measured 1.1e-3) and mean-rel stays 1e-5 (measured 5.5e-7)."""
    from transformers.integrations.mxfp4 import convert_moe_packed_tensors
    from transformers.models.gpt_oss.configuration_gpt_oss import GptOssConfig
    from transformers.models.gpt_oss.modeling_gpt_oss import GptOssMLP

    E, H, I, K, T = 4, 2880, 2880, 2, 8
    layer = synth.gptoss_layer(n_experts=E, hidden=H, inter=I, top_k=K, seed=7)
    cfg = GptOssConfig(hidden_size=H, intermediate_size=I, num_local_experts=E,
                       num_experts_per_tok=K, num_hidden_layers=1, num_attention_heads=4,
                       num_key_value_heads=1, head_dim=32, vocab_size=16)
    mlp = GptOssMLP(cfg).double().eval()
    x = synth.tokens(T, H, seed=9)
    with torch.no_grad():
        mlp.router.weight.copy_(_f64(layer.router_w))
        mlp.router.bias.copy_(_f64(layer.router_b))
        for name, blocks, scales in (("gate_up_proj", layer.gu_blocks, layer.gu_scales),
                                     ("down_proj", layer.dn_blocks, layer.dn_scales)):
            w = convert_moe_packed_tensors(torch.from_numpy(blocks), torch.from_numpy(scales),
                                           dtype=torch.float32)
            getattr(mlp.experts, name).copy_(w.double())
            del w
        mlp.experts.gate_up_proj_bias.copy_(_f64(layer.gu_bias))
        mlp.experts.down_proj_bias.copy_(_f64(layer.dn_bias))
        xt = torch.from_numpy(x.astype(np.float64))
        _, _, hf_idx = mlp.router(xt)
        hf_out, _ = mlp(xt[None])
    out, idx, _ = oracle.OracleMoe(layer).forward(x)
    np.testing.assert_array_equal(idx, hf_idx.numpy())
    _close(out, hf_out[0].numpy(), "GPT-OSS block, H = I = 2880", max_abs_bar=1e-2)


@pytest.mark.parametrize("E,H,I,K,max_abs_bar", [
    (8, 256, 256, 4, MAX_ABS),
    (4, 2048, 1792, 2, 1e-2),  # the LFM2.5 hidden and expert sizes
])
def test_lfm2_block_matches_transformers_lfm2_moe(E, H, I, K, max_abs_bar):
    from transformers.models.lfm2_moe.configuration_lfm2_moe import Lfm2MoeConfig
    from transformers.models.lfm2_moe.modeling_lfm2_moe import Lfm2MoeSparseMoeBlock

    T = 24
    layer = synth.lfm2_layer(n_experts=E, hidden=H, inter=I, top_k=K, seed=6)
    layer.sel_bias[:] = np.linspace(-0.02, 0.02, E, dtype=np.float32)
    cfg = Lfm2MoeConfig(hidden_size=H, moe_intermediate_size=I, num_experts=E,
                        num_experts_per_tok=K, norm_topk_prob=True, use_expert_bias=True,
                        routed_scaling_factor=1.0)
    blk = Lfm2MoeSparseMoeBlock(cfg).double().eval()

    def deq(raw, rows, k):
        return oracle.q4k_dequant(np.ascontiguousarray(raw).reshape(-1), rows * k).reshape(rows, k)

    gate = np.stack([deq(layer.gate_raw[e], I, H) for e in range(E)])
    up = np.stack([deq(layer.up_raw[e], I, H) for e in range(E)])
    down = np.stack([deq(layer.down_raw[e], H, I) for e in range(E)])
    x = synth.tokens(T, H, seed=7)
    with torch.no_grad():
        blk.gate.weight.copy_(torch.from_numpy(layer.router_w.astype(np.float64)))
        blk.expert_bias.copy_(torch.from_numpy(layer.sel_bias))
        blk.experts.gate_up_proj.copy_(torch.from_numpy(np.concatenate([gate, up], axis=1)))
        blk.experts.down_proj.copy_(torch.from_numpy(down))
        xt = torch.from_numpy(x.astype(np.float64))
        hf_idx, hf_w = blk.route_tokens_to_experts(blk.gate(xt))
        hf_out = blk(xt[None])
    out, idx, w = oracle.OracleLfm2(layer).forward(x)
    np.testing.assert_array_equal(idx, hf_idx.numpy())
    # transformers adds 1e-6 to the sum where the reference clamps it below at 1e-20
    np.testing.assert_allclose(w, hf_w.numpy(), rtol=2e-6, atol=1e-7)
    _close(out, hf_out[0].numpy(), f"LFM2.5 block H={H} I={I}", max_abs_bar=max_abs_bar)
