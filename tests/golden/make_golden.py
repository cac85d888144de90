"""Generate the golden fixtures under tests/golden/ from the REFERENCE code.

Run from the repo root, in a container where the reference checkout and
transformers 5.5.0 are importable:

    python tests/golden/make_golden.py --reference /path/to/reference

What each fixture pins, and which reference code produced it:

* ``q4_0_kat.npz`` - GGUF Q4_0 dequantisation by the reference's own
  ``GGUFLoader.dequantize_tensor`` (python/phantom/loader/gguf_loader.py:362-381,
  CPU branch), on the known-answer block of tests/audit_suite.py:36-41
  (nibbles 0x88, d = 1.5 -> zeros) and on 64 seeded random blocks.
* ``q4_k_ref.npz`` - GGUF Q4_K (and Q4_0) dequantisation by the reference's
  ``dequantize_tensor_cuda`` (gguf_loader.py:538-666, run with device="cpu"
  and target_dtype=float32, i.e. the fp32 values before the loader's bf16
  cast) - the function its model loader runs (gguf_loader.py:799) - on 48
  seeded random super-blocks; plus the same blocks through the reference's
  CPU ``GGUFLoader.dequantize_tensor`` Q4_K branch (gguf_loader.py:453-489),
  which orders the nibbles differently, and through the ``gguf`` package's
  ``quants.dequantize`` (llama.cpp's layout) when that package is present.
* ``router_phantom.npz`` - the reference's ``PhantomTopKRouter``
  (tests/test_moe_routing.py:43-72) on the shapes of its own
  ``test_router_correctness`` (x [2,4,256], 8 experts, top-2).
* ``qwen3_block_small.npz`` / ``mixtral_block_small.npz`` - transformers'
  ``Qwen3MoeSparseMoeBlock`` / ``MixtralSparseMoeBlock`` (the MoE code PHANTOM
  executes, python/phantom/phantom_cli.py:1393-1430) in fp32 on CPU, with
  expert weights set to the dequantised int4 values whose packed bytes are
  stored alongside.
* ``qwen2moe_block_small.npz`` - transformers' ``Qwen2MoeSparseMoeBlock``
  (routed experts + a sigmoid-gated shared expert of 4x the routed
  intermediate size, norm_topk_prob False) in fp32 on CPU, on the
  dequantised int4 values of the packed E + 4 experts stored alongside
  (routed experts, then the shared expert cut into 4 slices).
* ``deepseek_route.npz`` - transformers' ``DeepseekV3MoE.route_tokens_to_experts``
  (sigmoid scores, e_score_correction_bias, 16 experts in 4 groups, 2 groups
  kept, top-4, renormalised, routed_scaling_factor 2.5) on seeded fp32 logits.
* ``qwen3_cfg1.npz`` - the same Qwen3 block at BASELINE config 1 (H=2048,
  128 experts, top-8, I=768, T=16, fp32 inputs drawn from
  ``torch.Generator().manual_seed(0)``). The 320 MB of packed weights are
  not stored: the fixture keeps sha256 digests of the regenerated inputs and
  packed bytes, the block output, and the top-k indices/weights.

Only this generator touches the reference; the tests read the .npz files.
"""

from __future__ import annotations

import argparse
import hashlib
import logging
import sys
import types
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))
from oracle import moe_oracle as O  # noqa: E402

OUT = Path(__file__).resolve().parent


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def import_reference(ref: Path):
    # python/phantom/loader/safetensors_loader.py imports structlog unguarded;
    # a logging-backed stand-in lets the package import.
    sys.modules.setdefault("structlog", types.SimpleNamespace(
        get_logger=lambda *a, **k: logging.getLogger("phantom")))
    sys.path.insert(0, str(ref / "python"))
    sys.path.insert(0, str(ref / "tests"))
    from phantom.loader.gguf_loader import GGUFLoader, GGUFQuantType  # noqa: E402
    import test_moe_routing  # noqa: E402
    return GGUFLoader, GGUFQuantType, test_moe_routing


def make_q4_k(GGUFLoader, GGUFQuantType):
    from phantom.loader.gguf_loader import dequantize_tensor_cuda  # noqa: E402
    rng = np.random.default_rng(4321)
    nsb = 48
    d = (np.abs(rng.standard_normal(nsb)) * 2e-3).astype(np.float16)
    dmin = (np.abs(rng.standard_normal(nsb)) * 2e-3).astype(np.float16)
    sc = rng.integers(0, 256, size=(nsb, 12), dtype=np.uint8)
    qs = rng.integers(0, 256, size=(nsb, 128), dtype=np.uint8)
    raw = b"".join(d[i:i + 1].tobytes() + dmin[i:i + 1].tobytes() + sc[i].tobytes() + qs[i].tobytes()
                   for i in range(nsb))
    n = nsb * 256
    exe = dequantize_tensor_cuda(raw, GGUFQuantType.Q4_K, (n,), target_dtype=torch.float32, device="cpu").numpy()
    loader = GGUFLoader.__new__(GGUFLoader)
    cpu = loader.dequantize_tensor(raw, GGUFQuantType.Q4_K, (n,)).float().numpy()
    q40_d = (rng.standard_normal(32) * 0.01).astype(np.float16)
    q40_qs = rng.integers(0, 256, size=(32, 16), dtype=np.uint8)
    q40_raw = b"".join(q40_d[i:i + 1].tobytes() + q40_qs[i].tobytes() for i in range(32))
    q40 = dequantize_tensor_cuda(q40_raw, GGUFQuantType.Q4_0, (32 * 32,), target_dtype=torch.float32,
                                 device="cpu").numpy()
    extra = {}
    try:
        import gguf  # llama.cpp's own Python package
        extra["ggml"] = gguf.quants.dequantize(np.frombuffer(raw, dtype=np.uint8).reshape(nsb, 144),
                                               gguf.GGMLQuantizationType.Q4_K).reshape(-1).astype(np.float32)
    except Exception as e:  # pragma: no cover - optional cross-check
        print("gguf package cross-check skipped:", e)
    np.savez_compressed(OUT / "q4_k_ref.npz", raw=np.frombuffer(raw, dtype=np.uint8), out_f32=exe,
                        out_cpu_branch_bf16=cpu, q4_0_raw=np.frombuffer(q40_raw, dtype=np.uint8),
                        q4_0_out_f32=q40, **extra)


def make_q4_0(GGUFLoader, GGUFQuantType):
    loader = GGUFLoader.__new__(GGUFLoader)
    # audit_suite.py:36-41 known answer
    kat_raw = np.array([1.5], dtype=np.float16).tobytes() + bytes([0x88] * 16)
    kat_out = loader.dequantize_tensor(kat_raw, GGUFQuantType.Q4_0, (32,)).float().numpy()
    rng = np.random.default_rng(1234)
    n_blocks = 64
    d = (rng.standard_normal(n_blocks) * 0.01).astype(np.float16)
    qs = rng.integers(0, 256, size=(n_blocks, 16), dtype=np.uint8)
    raw = b"".join(d[i:i + 1].tobytes() + qs[i].tobytes() for i in range(n_blocks))
    out = loader.dequantize_tensor(raw, GGUFQuantType.Q4_0, (n_blocks * 32,)).float().numpy()
    np.savez_compressed(OUT / "q4_0_kat.npz",
                        kat_raw=np.frombuffer(kat_raw, dtype=np.uint8), kat_out=kat_out,
                        raw=np.frombuffer(raw, dtype=np.uint8), out_bf16=out)


def make_router_phantom(tmr):
    torch.manual_seed(7)
    router = tmr.PhantomTopKRouter(256, 8, 2)
    x = torch.randn(2, 4, 256)
    with torch.no_grad():
        w, idx = router(x)
    np.savez_compressed(OUT / "router_phantom.npz", x=x.numpy(), gate=router.gate.weight.detach().numpy(),
                        weights=w.numpy(), indices=idx.numpy().astype(np.int32))


def _tf_block(kind: str, H, E, k, I, renorm=True):
    if kind == "qwen3":
        from transformers.models.qwen3_moe.configuration_qwen3_moe import Qwen3MoeConfig
        from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeSparseMoeBlock
        cfg = Qwen3MoeConfig(hidden_size=H, num_experts=E, num_experts_per_tok=k,
                             moe_intermediate_size=I, norm_topk_prob=renorm)
        cfg._experts_implementation = "eager"
        return Qwen3MoeSparseMoeBlock(cfg).eval()
    from transformers.models.mixtral.configuration_mixtral import MixtralConfig
    from transformers.models.mixtral.modeling_mixtral import MixtralSparseMoeBlock
    cfg = MixtralConfig(hidden_size=H, num_local_experts=E, num_experts_per_tok=k, intermediate_size=I)
    cfg._experts_implementation = "eager"
    return MixtralSparseMoeBlock(cfg).eval()


def run_tf_block(kind, x, wr, d13, d2, k, renorm=True):
    E, I2, H = d13.shape
    blk = _tf_block(kind, H, E, k, I2 // 2, renorm)
    with torch.no_grad():
        blk.gate.weight.copy_(torch.from_numpy(wr))
        blk.experts.gate_up_proj.copy_(torch.from_numpy(d13))
        blk.experts.down_proj.copy_(torch.from_numpy(d2))
        xt = torch.from_numpy(x)
        probs, scores, idx = blk.gate(xt)
        out = blk(xt[None])
        if isinstance(out, tuple):
            out = out[0]
    return (out[0].numpy().astype(np.float32), probs.numpy().astype(np.float32),
            idx.numpy().astype(np.int32), scores.numpy().astype(np.float32))


def small_block_inputs(T, H, E, I, seed):
    """Seeded inputs of a small-block fixture (tests regenerate the dense
    expert weights this way instead of storing them)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, H, generator=g).numpy()
    wr = (torch.randn(E, H, generator=g) * 0.02).numpy()
    w13 = (torch.randn(E, 2 * I, H, generator=g) * 0.02).numpy()
    w2 = (torch.randn(E, H, I, generator=g) * 0.02).numpy()
    return x, wr, w13, w2


def make_small_block(kind, name, T, H, E, k, I, group, seed):
    x, wr, w13, w2 = small_block_inputs(T, H, E, I, seed)
    p13, s13 = O.quantize_int4(w13, group)
    p2, s2 = O.quantize_int4(w2, group)
    d13 = O.dequantize_int4(p13, s13, group)
    d2 = O.dequantize_int4(p2, s2, group)
    out, probs, idx, scores = run_tf_block(kind, x, wr, d13, d2, k)
    np.savez_compressed(OUT / name, x=x, wr=wr, w13_q=p13, w13_s=s13, w2_q=p2, w2_s=s2,
                        dims=np.array([T, H, E, I, seed], np.int32), group=np.int32(group),
                        top_k=np.int32(k), out=out, probs=probs, idx=idx, scores=scores)


def make_qwen2moe_block(name, T, H, E, k, I, m, group, seed):
    from transformers.models.qwen2_moe.configuration_qwen2_moe import Qwen2MoeConfig
    from transformers.models.qwen2_moe.modeling_qwen2_moe import Qwen2MoeSparseMoeBlock
    x, wr, w13, w2 = small_block_inputs(T, H, E, I, seed)
    g = torch.Generator().manual_seed(seed + 1000)
    Is = m * I
    sgp = (torch.randn(Is, H, generator=g) * 0.02).numpy()
    sup = (torch.randn(Is, H, generator=g) * 0.02).numpy()
    sdp = (torch.randn(H, Is, generator=g) * 0.02).numpy()
    sgate = (torch.randn(1, H, generator=g) * 0.05).numpy()
    # shared expert cut into m experts of size I, after the routed ones
    s13 = np.concatenate([sgp.reshape(m, I, H), sup.reshape(m, I, H)], axis=1)
    s2 = sdp.reshape(H, m, I).transpose(1, 0, 2)
    p13, q13 = O.quantize_int4(np.concatenate([w13, s13]).astype(np.float32), group)
    p2, q2 = O.quantize_int4(np.concatenate([w2, s2]).astype(np.float32), group)
    d13, d2 = O.dequantize_int4(p13, q13, group), O.dequantize_int4(p2, q2, group)
    cfg = Qwen2MoeConfig(hidden_size=H, num_experts=E, num_experts_per_tok=k, moe_intermediate_size=I,
                         shared_expert_intermediate_size=Is, norm_topk_prob=False)
    cfg._experts_implementation = "eager"
    blk = Qwen2MoeSparseMoeBlock(cfg).eval()
    with torch.no_grad():
        blk.gate.weight.copy_(torch.from_numpy(wr))
        blk.experts.gate_up_proj.copy_(torch.from_numpy(d13[:E]))
        blk.experts.down_proj.copy_(torch.from_numpy(d2[:E]))
        blk.shared_expert.gate_proj.weight.copy_(torch.from_numpy(d13[E:, :I].reshape(Is, H)))
        blk.shared_expert.up_proj.weight.copy_(torch.from_numpy(d13[E:, I:].reshape(Is, H)))
        blk.shared_expert.down_proj.weight.copy_(torch.from_numpy(d2[E:].transpose(1, 0, 2).reshape(H, Is)))
        blk.shared_expert_gate.weight.copy_(torch.from_numpy(sgate))
        xt = torch.from_numpy(x)
        _, scores, idx = blk.gate(xt)
        out = blk(xt[None])[0]
    np.savez_compressed(OUT / name, x=x, wr=wr, w13_q=p13, w13_s=q13, w2_q=p2, w2_s=q2, shared_gate=sgate,
                        dims=np.array([T, H, E, I, m, seed], np.int32), group=np.int32(group),
                        top_k=np.int32(k), out=out.numpy().astype(np.float32),
                        idx=idx.numpy().astype(np.int32), scores=scores.numpy().astype(np.float32))


def make_deepseek_route(name, T=64, E=16, n_group=4, topk_group=2, k=4, scale=2.5, seed=15):
    from transformers.models.deepseek_v3.configuration_deepseek_v3 import DeepseekV3Config
    from transformers.models.deepseek_v3.modeling_deepseek_v3 import DeepseekV3MoE
    cfg = DeepseekV3Config(hidden_size=64, n_routed_experts=E, n_group=n_group, topk_group=topk_group,
                           num_experts_per_tok=k, moe_intermediate_size=32, n_shared_experts=1,
                           routed_scaling_factor=scale, norm_topk_prob=True)
    moe = DeepseekV3MoE(cfg).eval()
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(T, E, generator=g) * 2.0
    bias = torch.randn(E, generator=g) * 0.1
    with torch.no_grad():
        moe.gate.e_score_correction_bias.copy_(bias)
        idx, w = moe.route_tokens_to_experts(logits)
    np.savez_compressed(OUT / name, logits=logits.numpy(), bias=bias.numpy(), idx=idx.numpy().astype(np.int32),
                        w=w.numpy().astype(np.float32), cfg=np.array([E, n_group, topk_group, k], np.int32),
                        scale=np.float32(scale))


def gen_cfg1_inputs():
    """BASELINE config 1 inputs (documented procedure; the GPU tests repeat it)."""
    g = torch.Generator().manual_seed(0)
    T, H, E, I = 16, 2048, 128, 768
    x = torch.randn(T, H, generator=g)
    wr = torch.randn(E, H, generator=g) * 0.02
    w13 = torch.randn(E, 2 * I, H, generator=g) * 0.02
    w2 = torch.randn(E, H, I, generator=g) * 0.02
    return x, wr, w13, w2


def make_cfg1():
    x, wr, w13, w2 = gen_cfg1_inputs()
    E = w13.shape[0]
    p13 = np.empty((E, w13.shape[1], w13.shape[2] // 2), np.uint8)
    s13 = np.empty((E, w13.shape[1], w13.shape[2] // 64), np.float16)
    p2 = np.empty((E, w2.shape[1], w2.shape[2] // 2), np.uint8)
    s2 = np.empty((E, w2.shape[1], w2.shape[2] // 64), np.float16)
    for e in range(E):
        p13[e], s13[e] = O.quantize_int4(w13[e].numpy(), 64)
        p2[e], s2[e] = O.quantize_int4(w2[e].numpy(), 64)
    d13 = np.stack([O.dequantize_int4(p13[e], s13[e]) for e in range(E)])
    d2 = np.stack([O.dequantize_int4(p2[e], s2[e]) for e in range(E)])
    out, probs, idx, scores = run_tf_block("qwen3", x.numpy(), wr.numpy(), d13, d2, 8)
    np.savez_compressed(
        OUT / "qwen3_cfg1.npz", out=out, probs=probs, idx=idx, scores=scores,
        sha_x=sha(x.numpy()), sha_wr=sha(wr.numpy()), sha_w13_q=sha(p13), sha_w13_s=sha(s13),
        sha_w2_q=sha(p2), sha_w2_s=sha(s2))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    ap.add_argument("--skip-cfg1", action="store_true", help="keep the existing qwen3_cfg1.npz")
    ap.add_argument("--only", choices=["q4_k", "qwen2moe", "deepseek"], help="regenerate one fixture only")
    args = ap.parse_args()
    GGUFLoader, QT, tmr = import_reference(Path(args.reference))
    if args.only == "q4_k":
        make_q4_k(GGUFLoader, QT)
        return
    if args.only == "deepseek":
        make_deepseek_route("deepseek_route.npz")
        return
    if args.only == "qwen2moe":
        make_qwen2moe_block("qwen2moe_block_small.npz", T=10, H=256, E=8, k=2, I=128, m=4, group=64, seed=14)
        return
    make_q4_0(GGUFLoader, QT)
    make_q4_k(GGUFLoader, QT)
    make_router_phantom(tmr)
    make_small_block("qwen3", "qwen3_block_small.npz", T=12, H=256, E=16, k=4, I=128, group=64, seed=11)
    make_small_block("qwen3", "qwen3_block_small_g32.npz", T=9, H=256, E=8, k=2, I=64, group=32, seed=12)
    make_small_block("mixtral", "mixtral_block_small.npz", T=10, H=256, E=8, k=2, I=128, group=64, seed=13)
    make_qwen2moe_block("qwen2moe_block_small.npz", T=10, H=256, E=8, k=2, I=128, m=4, group=64, seed=14)
    make_deepseek_route("deepseek_route.npz")
    if not args.skip_cfg1:
        make_cfg1()
    for p in sorted(OUT.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
