"""The ``<op>_BEST.py`` plugin modules under the reference's own loader rules.

Discovery and loading follow ``extra_bench.py:24-27`` (importlib by path,
``launch_kernel`` attribute) and ``extra_bench.py:65-70`` (file name ->
operator name), restated here.
"""

import glob
import importlib.util
import os

import pytest
import torch

import chia_proj_b200 as cp
import oracle

PLUGINS = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                       "chia_proj_b200", "plugins")


def discover():
    found = {}
    for p in glob.glob(os.path.join(PLUGINS, "*_BEST.py")):
        bn = os.path.basename(p).replace("_BEST.py", "")
        op = "sigmoid_attn" if bn.startswith("sigmoid_") else bn.split("_gemini")[0]
        found.setdefault(op, []).append(p)
    return found


def load(p):
    sp = importlib.util.spec_from_file_location("k" + str(abs(hash(p))), p)
    m = importlib.util.module_from_spec(sp)
    sp.loader.exec_module(m)
    return m.launch_kernel


def test_every_operator_has_one_plugin(lib):
    found = discover()
    assert sorted(found) == sorted(cp.OPS)
    for op, paths in found.items():
        assert len(paths) == 1
        assert callable(load(paths[0]))


@pytest.mark.gpu
@pytest.mark.parametrize("op", sorted(cp.OPS))
def test_plugin_runs_reference_shape(cuda, op):
    """The reference's Table-2 shape [2,32,2048,128] bf16 (extra_bench.py:79-81),
    gated with its relative-error rule (extra_bench.py:29,121) on two heads."""
    fn = load(discover()[op][0])
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(2, 32, 2048, 128, generator=g).to(torch.bfloat16) for _ in range(3))
    out = fn(q.cuda(), k.cuda(), v.cuda())
    assert out.shape == q.shape and out.dtype == q.dtype
    o = out[:, :2].float().cpu()
    # per-head parameters depend on H=32: give the oracle those of heads 0 and 1
    kw = {}
    if op == "bias_alibi":
        kw = {"slopes": cp.reference_alibi_slopes(32)[:2]}
    elif op == "temp_perhead":
        kw = {"temps": cp.reference_temps(32)[:2]}
    ref = oracle.run_op(op, q[:, :2], k[:, :2], v[:, :2], **kw)
    rel = (o - ref).abs().max().item() / (ref.abs().max().item() + 1e-6)
    assert rel < 3e-2, (op, rel)
    assert (o - ref).abs().max().item() <= 2e-2 * max(1.0, ref.abs().max().item())


def test_plugins_load_from_a_reference_style_directory(lib, tmp_path):
    """A reference checkout picks the plugins up from a ``kernels_gemini*``
    directory of symlinks (``extra_bench.py:65-70``); loaded from there in a
    fresh interpreter, each one still finds this package."""
    import subprocess
    import sys
    d = tmp_path / "kernels_gemini_b200"
    d.mkdir()
    for p in glob.glob(os.path.join(PLUGINS, "*_BEST.py")):
        os.symlink(p, d / os.path.basename(p))
    prog = (
        "import glob, importlib.util, os\n"
        "n = 0\n"
        "for p in glob.glob(os.path.join('kernels_gemini*', '*_BEST.py')):\n"
        "    sp = importlib.util.spec_from_file_location('k' + str(abs(hash(p))), p)\n"
        "    m = importlib.util.module_from_spec(sp); sp.loader.exec_module(m)\n"
        "    assert callable(m.launch_kernel); n += 1\n"
        "print(n)\n")
    env = {k: v for k, v in os.environ.items() if k != "PYTHONPATH"}
    out = subprocess.run([sys.executable, "-c", prog], cwd=tmp_path, env=env,
                         capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    assert out.stdout.strip() == str(len(cp.OPS))
