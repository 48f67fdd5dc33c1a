"""Pins the oracle's sparse-MoE FFN (oracle/fence_oracle.c moe_ffn, which every MoE parity test of
the engine is checked against) to a published implementation of the same algorithm: the Mixtral
sparse-MoE block of Hugging Face transformers (MixtralSparseMoeBlock: softmax over the router
logits, top-k, renormalised; each chosen expert's down(silu(gate x) * up x) weighted and summed).
The reference has no expert tensors, so this is the only outside anchor for config 4's routing.

Both run on the same seeded inputs with the same weights: the GGUF's Q6_K / Q8_0 expert matrices
dequantised (Q6_K by the oracle's dequantiser, itself pinned to the reference's host oracle;
Q8_0 is one fp16 scale times 32 int8s) and the fp32 router. transformers runs in float64. The
oracle keeps the reference's numerics points: fp32 activations, and for Q6_K linears inputs
rounded to fp16 (qwen3.cu:278-336); the bound covers that rounding of the SwiGLU output, the
only input the two sides do not share. CPU only."""
import numpy as np
import pytest

import gguf_py

torch = pytest.importorskip("torch")
mixtral = pytest.importorskip("transformers.models.mixtral.modeling_mixtral")
MixtralConfig = pytest.importorskip("transformers").MixtralConfig


def _dequant(orc, raw: bytes, ty: int, rows: int, cols: int) -> np.ndarray:
    b = np.frombuffer(raw, np.uint8)
    if ty == 8:  # Q8_0
        blk = b.reshape(-1, 34)
        d = blk[:, :2].copy().view(np.float16).astype(np.float64)
        q = blk[:, 2:].view(np.int8).astype(np.float64)
        return (d * q).reshape(rows, cols)
    assert ty == 14, ty  # Q6_K
    blk = np.ascontiguousarray(b.reshape(-1, 210))
    out = np.empty((blk.shape[0], 256), np.float64)
    import ctypes
    for i in range(blk.shape[0]):
        orc.oracle().oracle_q6k_dequant(blk[i].ctypes.data_as(ctypes.c_void_p), out[i].ctypes.data_as(ctypes.c_void_p))
    return out.reshape(rows, cols)


def _hf_block(orc, rd, layer, H, F, E, K):
    cfg = MixtralConfig(hidden_size=H, intermediate_size=F, num_local_experts=E, num_experts_per_tok=K,
                        hidden_act="silu", router_jitter_noise=0.0)
    blk = mixtral.MixtralSparseMoeBlock(cfg).double().eval()
    p = f"blk.{layer}."
    dims, ty, _ = rd.tensors[p + "ffn_gate_inp.weight"]
    assert ty == 0 and dims == [H, E]
    router = np.frombuffer(rd.tensor_bytes(p + "ffn_gate_inp.weight"), np.float32).reshape(E, H)
    gate = _dequant(orc, rd.tensor_bytes(p + "ffn_gate_exps.weight"), rd.tensors[p + "ffn_gate_exps.weight"][1],
                    E * F, H).reshape(E, F, H)
    up = _dequant(orc, rd.tensor_bytes(p + "ffn_up_exps.weight"), rd.tensors[p + "ffn_up_exps.weight"][1],
                  E * F, H).reshape(E, F, H)
    down = _dequant(orc, rd.tensor_bytes(p + "ffn_down_exps.weight"), rd.tensors[p + "ffn_down_exps.weight"][1],
                    E * H, F).reshape(E, H, F)
    with torch.no_grad():
        blk.gate.weight.copy_(torch.from_numpy(router.astype(np.float64)))
        blk.experts.gate_up_proj.copy_(torch.from_numpy(np.concatenate([gate, up], axis=1)))
        blk.experts.down_proj.copy_(torch.from_numpy(down))
    return blk, router.astype(np.float64)


@pytest.mark.parametrize("cfg,k", [("tiny-moe", 2), ("tiny-moe", 1), ("tiny-moe-q8", 2), ("tiny-moe-q8", 1)])
def test_oracle_moe_block_matches_transformers_mixtral(fb, orc, tmp_path, cfg, k):
    path = str(tmp_path / f"{cfg}.gguf")
    fb.synth_write(path, cfg, seed=43, n_experts_used=k)
    om = orc.OracleModel(path, max_ctx=64, kv_bf16=False)
    H, F, E = om.embed_dim, om.ff_dim, om.n_experts
    assert om.n_experts_used == k
    q6 = om.linear_type == 14
    rd = gguf_py.Reader(path)
    rng = np.random.default_rng(5)
    checked = 0
    for layer in range(om.n_layers):
        blk, router = _hf_block(orc, rd, layer, H, F, E, k)
        for _ in range(12):
            x = rng.standard_normal(H).astype(np.float32)
            if q6:  # the Q6_K linears see fp16 inputs on both sides
                x = x.astype(np.float16).astype(np.float32)
            logits = router @ x.astype(np.float64)
            srt = np.sort(logits)[::-1]
            if srt[k - 1] - srt[k] < 1e-6:  # a routing near-tie: either choice is right
                continue
            got, sel = om.moe_ffn(layer, x)
            with torch.no_grad():
                _, _, idx = blk.gate(torch.from_numpy(x.astype(np.float64))[None])
                want = blk(torch.from_numpy(x.astype(np.float64))[None, None]).numpy().reshape(H)
            assert list(sel[:k]) == [int(i) for i in idx[0]], (layer, sel, idx)
            scale = np.abs(want).max()
            err = np.abs(got.astype(np.float64) - want).max()
            bound = (1e-3 if q6 else 2e-6) * scale  # Q6_K: fp16 rounding of the SwiGLU output before down
            assert err <= bound, (layer, err, scale)
            checked += 1
    om.close()
    assert checked >= 16
