"""The reference's own validation scripts, run against this build.

co_alibi_attn/benchmark_fwd_pass.py and benchmark_bwd_pass.py (B1 H16 S4096 D128
bf16) compare ``co_alibi_attention`` with a PyTorch restatement on the GPU and print
``passed: <name> diff=...`` or ``WARNING: <name> Error: ...`` (their
``assert_similar``, 1 - calc_sim <= 1e-4).  As files they put their own checkout
first on sys.path; loaded as modules after this build's ``co_alibi_attn`` is
imported, their ``from co_alibi_attn import co_alibi_attention`` resolves to this
build, and their ``main()`` runs unchanged.  The scripts come from the unmodified
reference package installed in baseline/_ref (baseline/install_ref.py); the test
skips when it is absent."""
import importlib.util
import os

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_PKG = os.path.join(ROOT, "baseline", "_ref", "co_alibi_attn")


def _load(name):
    path = os.path.join(REF_PKG, name + ".py")
    if not os.path.exists(path):
        pytest.skip("baseline/_ref holds no reference package (python baseline/install_ref.py <checkout>)")
    import co_alibi_attn  # this build's package, so the script's import finds it in sys.modules
    spec = importlib.util.spec_from_file_location("reference_" + name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    assert mod.co_alibi_attention is co_alibi_attn.co_alibi_attention, "the script imported another package"
    return mod


@pytest.mark.parametrize("script,names", [
    ("benchmark_fwd_pass", ["output"]),
    ("benchmark_bwd_pass", ["dq", "dk", "dv"]),
])
def test_reference_validation_script(script, names, capsys):
    mod = _load(script)
    mod.main()
    out = capsys.readouterr().out
    assert "Error" not in out, out[-2000:]
    for n in names:
        assert f"passed: {n} diff=" in out, out[-2000:]
