"""GPU: the reference package itself runs on top of ksdraft_b200.install().

The unmodified reference (curvedinf/ksdraft, installed with pip into
baseline/_ref, which travels with the repository) is imported in a child
interpreter after install(); no Triton kernel may launch (Triton's JIT entry
is replaced by one that raises).  The checks restate the reference's own
test cases for the int8 tier (tests/test_int8.py: quantiser error bound,
padding, zero rows, GEMM parity with the fp32 tier at rtol 1e-4 / atol 1e-3,
Int8Linear within 5% of fp32) and for Rosa (tests/test_rosa.py: the hand
case, random short streams against a brute force, no match), then run a
small KSDraftModel through to_int8 (the reference's to_int8 cases: eval
forward within 15% of fp32, training gradients flowing), the reference Trainer
(warm-up stage, T = 32 so its CUDA Rosa credit path applies) and
export / load_export with weights this build's training step produced."""

import subprocess
import sys
import textwrap
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / "baseline" / "_ref"

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not (REF / "ksdraft" / "__init__.py").exists(),
                                 reason="the reference is not installed in baseline/_ref")]

PRELUDE = f"""
import sys
sys.path[:0] = [{str(ROOT)!r}, {str(REF)!r}]
import triton.runtime.jit as _jit

def _no_triton(*a, **k):
    raise RuntimeError("a Triton kernel was launched")
_jit.JITFunction.run = _no_triton
import ksdraft_b200.install as kb
done = kb.install()
import torch
import ksdraft
assert ksdraft.__file__.startswith({str(REF)!r}), ksdraft.__file__
"""


def _child(code: str, timeout=600) -> str:
    r = subprocess.run([sys.executable, "-c", PRELUDE + textwrap.dedent(code)],
                       capture_output=True, text=True, timeout=timeout, cwd=str(ROOT))
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-6000:]
    return r.stdout


def test_reference_int8_cases_on_ksdraft_b200():
    out = _child("""
        from ksdraft.kernels.quant import quantize_last_dim, dequantize_last_dim
        from ksdraft.kernels.gemm import w8a8_gemm
        from ksdraft.kernels.linear import Int8Linear
        import ksdraft.kernels.gemm as G
        assert G.__name__ == "ksdraft_b200.kernels.gemm", G.__name__
        dev = "cuda"
        g = torch.Generator().manual_seed(0)
        # quantiser: error within half a step, padding, zero rows
        x = torch.randn(64, 300, generator=g)
        c, s = quantize_last_dim(x.to(dev))
        assert c.shape == (64, 300) and s.shape == (64, 3)
        err = (dequantize_last_dim(c, s).cpu() - x).abs()
        step = s.float().cpu().repeat_interleave(128, 1)[:, :300]
        assert bool((err <= step / 2 + 1e-6).all())
        z, zs = quantize_last_dim(torch.zeros(2, 128, device=dev))
        assert int(z.abs().sum()) == 0
        # GEMM against the fp32 tier (dequantise, then matmul) at rtol 1e-4 / atol 1e-3
        for M, K, N in ((16, 256, 128), (64, 128, 96), (33, 384, 64), (128, 128, 128)):
            a = torch.randn(M, K, generator=g)
            w = torch.randn(N, K, generator=g) * 0.1
            ac, as_ = quantize_last_dim(a.to(dev))
            wc, ws = quantize_last_dim(w.to(dev))
            y = w8a8_gemm(ac, as_, wc, ws).cpu()
            ref = dequantize_last_dim(ac, as_).cpu() @ dequantize_last_dim(wc, ws).cpu().T
            assert torch.allclose(y, ref, rtol=1e-4, atol=1e-3), (M, K, N)
        # Int8Linear against fp32
        lin = torch.nn.Linear(256, 96).to(dev)
        q = Int8Linear.from_float(lin).eval()
        xx = torch.randn(48, 256, device=dev)
        with torch.no_grad():
            rel = ((q(xx) - lin(xx)).norm() / lin(xx).norm()).item()
        assert rel < 0.05, rel
        print("int8 ok", rel)
    """)
    assert "int8 ok" in out


def test_reference_rosa_cases_on_ksdraft_b200():
    out = _child("""
        import itertools, random
        from ksdraft.model.rosa import _match_payload_sign
        import ksdraft.model.rosa as R
        assert R._match_payload_sign.__module__ == "ksdraft_b200.model.rosa"
        dev = "cuda"
        t = lambda l: torch.tensor([l], dtype=torch.int8, device=dev)
        s = _match_payload_sign(t([0, 1, 1, 1]), t([1, 0, 1, 1]), t([1, 0, 0, 1]))
        assert s.cpu().tolist() == [[-1.0, -1.0, -1.0, 1.0]], s

        def brute(q, k, v):
            T = len(q)
            out = []
            for tt in range(T):
                best, bj = 0, -1
                for j in range(tt):
                    L = 0
                    while L <= j and q[tt - L] == k[j - L] and L < min(62, T - 1):
                        L += 1
                    if L > 0 and L >= best:
                        best, bj = L, j
                out.append(1.0 if bj >= 0 and v[bj + 1] else -1.0)
            return out
        rng = random.Random(5)
        for _ in range(20):
            T = rng.randint(1, 24)
            q, k, v = ([rng.randint(0, 1) for _ in range(T)] for _ in range(3))
            got = _match_payload_sign(t(q), t(k), t(v)).cpu().tolist()[0]
            assert got == brute(q, k, v), (q, k, v, got)
        none = _match_payload_sign(t([1, 1, 1]), t([0, 0, 0]), t([1, 1, 1]))
        assert none.cpu().tolist() == [[-1.0, -1.0, -1.0]]
        print("rosa ok")
    """)
    assert "rosa ok" in out


def test_reference_model_trainer_and_export_on_ksdraft_b200(tmp_path):
    out = _child(f"""
        from ksdraft.config import KSDraftConfig
        from ksdraft.model import KSDraftModel
        from ksdraft.model.int8_convert import to_int8
        from ksdraft.train import Trainer, TrainConfig, WindowSampler
        from ksdraft.export import export_model, load_export
        from ksdraft_b200.train.draft_step import DraftShape, DraftTrainStep
        dev = "cuda"
        # the reference's own to_int8 cases (tests/test_int8_convert.py), restated:
        # a "woken" tiny model (head, out_proj and KS3 up drawn), eval forward
        # within 15% of the float model, and training gradients that flow
        tiny = KSDraftConfig(vocab_size=256, layers=2, d_model=96, head_size=32,
                             rosa_streams=32, ks3_charts=64)
        torch.manual_seed(0)
        model = KSDraftModel(tiny).eval()
        with torch.no_grad():
            model.head.weight.normal_(0, 0.02)
            for blk in model.blocks:
                blk.rosa.out_proj.weight.normal_(0, 0.05)
                blk.ffn.up.weight.normal_(0, 0.05)
        model = model.to(dev)
        tokens = torch.randint(0, 256, (2, 16), device=dev)
        with torch.no_grad():
            y_ref, _ = model(tokens)
            y_q, _ = to_int8(model)(tokens)
        rel = ((y_q - y_ref).norm() / y_ref.norm()).item()
        assert torch.isfinite(y_q).all() and rel < 0.15, rel
        torch.manual_seed(0)
        wm = KSDraftModel(tiny, teacher_dim=96).train()
        with torch.no_grad():
            wm.head.weight.normal_(0, 0.02)
            for blk in wm.blocks:
                blk.rosa.out_proj.weight.normal_(0, 0.05)
                blk.ffn.up.weight.normal_(0, 0.05)
        conv = to_int8(wm.to(dev))
        toks = torch.randint(0, 256, (2, 8), device=dev)
        logits, _ = conv(toks, teacher_states=torch.randn(2, 8, 96, device=dev))
        torch.nn.functional.cross_entropy(logits[:, :-1].flatten(0, 1),
                                          toks[:, 1:].flatten()).backward()
        grads = [p.grad for p in conv.parameters() if p.grad is not None]
        assert grads and all(torch.isfinite(g).all() for g in grads)
        qg = conv.blocks[0].rosa.q_proj.weight.grad        # the CUDA credit path
        assert qg is not None and torch.isfinite(qg).all()
        cfg = KSDraftConfig(vocab_size=512, layers=2, d_model=128, rosa_streams=64,
                            ks3_charts=256)
        q = to_int8(KSDraftModel(cfg, device=dev))
        # the reference trainer, warm-up stage, on the int8 model (T = 32: the CUDA
        # Rosa training path with its counterfactual credits applies)
        ids = torch.randint(0, 512, (4096,)).tolist()
        tr = Trainer(q.train(), None, WindowSampler(ids, 32, seed=1),
                     TrainConfig(steps=2, seq_len=32, batch_size=2), device=dev)
        hist = tr.train("warmup", log=lambda *a: None)
        assert all(map(lambda r: r["loss"] == r["loss"], hist["history"]))
        # export / load_export of weights trained by this build's full step
        shape = DraftShape(vocab=512, layers=2, d_model=128, streams=64, charts=256,
                           teacher_dim=64)
        st = DraftTrainStep(shape, dev, seed=3, act_dtype=torch.float32)
        tok = torch.randint(0, 512, (2, 33), device=dev)
        st(tok, torch.randn(2, 32, 64, device=dev))
        ref_model = KSDraftModel(cfg, teacher_dim=64)
        sd = {{k: v.detach().cpu() for k, v in st.parameter_dict().items()}}
        sd["head.weight"] = sd["embedding.weight"]
        ref_model.load_state_dict(sd)
        export_model(ref_model, {str(tmp_path)!r})
        back = load_export({str(tmp_path)!r})
        for k, v in st.parameter_dict().items():
            assert torch.equal(back.state_dict()[k], v.detach().cpu()), k
        print("model ok", rel)
    """)
    assert "model ok" in out
