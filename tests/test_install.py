"""ksdraft_b200.install rebinds a `ksdraft` package's hot path (CPU only).

A stand-in package with the reference's module layout and import statements
(ksdraft/kernels/__init__.py:7-8 style `from .quant import ...`) is written to
a temporary directory and imported in a child interpreter."""

import subprocess
import sys
import textwrap
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]

FILES = {
    "ksdraft/__init__.py": "",
    "ksdraft/kernels/__init__.py":
        "from .quant import GROUP_SIZE, quantize_last_dim, dequantize_last_dim\n"
        "from .linear import Int8Linear\n",
    "ksdraft/kernels/quant.py": "GROUP_SIZE = 128\nquantize_last_dim = 'reference'\n"
                                "dequantize_last_dim = 'reference'\n",
    "ksdraft/kernels/gemm.py": "w8a8_gemm = 'reference'\n",
    "ksdraft/kernels/linear.py": "Int8Linear = 'reference'\n",
    "ksdraft/kernels/ks3_int8.py": "KS3Int8Cell = 'reference'\n",
    "ksdraft/kernels/ks3_triton.py": "project_fused = 'reference'\n",
    "ksdraft/kernels/rosa_credit_gpu.py": "MAX_WINDOW = 63\nHardRosaGPU = 'reference'\n",
    "ksdraft/model/__init__.py": "",
    "ksdraft/model/rosa.py":
        "_match_payload_sign = 'reference'\n"
        "class RosaMixer:\n"
        "    def forward(self, *a):\n"
        "        return _match_payload_sign\n",
    "ksdraft/train/__init__.py": "",
    "ksdraft/train/stages.py": "quantize_last_dim_dithered = 'reference'\n"
                               "def wtv_loss():\n    return 'kept'\n",
}


def _write(tmp_path):
    for rel, text in FILES.items():
        p = tmp_path / rel
        p.parent.mkdir(parents=True, exist_ok=True)
        p.write_text(text)


def _run(tmp_path, code):
    env_code = f"import sys; sys.path[:0] = [{str(ROOT)!r}, {str(tmp_path)!r}]\n" + code
    r = subprocess.run([sys.executable, "-c", env_code], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    return r.stdout


def test_install_rebinds_modules_and_functions(tmp_path):
    _write(tmp_path)
    out = _run(tmp_path, textwrap.dedent("""
        import ksdraft_b200.install as kb
        done = kb.install()
        import ksdraft.kernels as K
        import ksdraft.kernels.gemm as G
        from ksdraft.kernels.ks3_int8 import KS3Int8Cell
        from ksdraft.model import rosa
        from ksdraft.train import stages
        import ksdraft_b200.kernels.quant as q
        import ksdraft_b200.kernels.gemm as g
        import ksdraft_b200.kernels.ks3_int8 as k
        import ksdraft_b200.model.rosa as r
        import ksdraft_b200.train.stages as s
        assert K.quantize_last_dim is q.quantize_last_dim
        assert K.quant is q and G is g and G.w8a8_gemm is g.w8a8_gemm
        assert KS3Int8Cell is k.KS3Int8Cell
        assert rosa._match_payload_sign is r._match_payload_sign
        assert rosa.RosaMixer().forward() is r._match_payload_sign   # looked up at call time
        assert stages.quantize_last_dim_dithered is s.quantize_last_dim_dithered
        assert stages.wtv_loss() == 'kept'                             # rest untouched
        import ksdraft.kernels.rosa_credit_gpu as cg
        import ksdraft_b200.kernels.rosa_credit_gpu as mine
        assert cg is mine and cg.HardRosaGPU is mine.HardRosaGPU      # the whole module
        print(len(done))
    """))
    assert out.strip() == "8"


def test_install_refuses_after_reference_import(tmp_path):
    _write(tmp_path)
    out = _run(tmp_path, textwrap.dedent("""
        import ksdraft.kernels
        import ksdraft_b200.install as kb
        try:
            kb.install()
        except RuntimeError as e:
            print('refused:', e)
    """))
    assert "refused:" in out and "ksdraft.kernels.quant" in out
