"""Install the unmodified reference package into baseline/_ref (git-ignored).

    python baseline/install_ref.py <reference checkout root>

The reference checkout has neither setup.py nor pyproject.toml, so the offline
``pip install --target baseline/_ref <checkout>`` fails ("Neither 'setup.py' nor
'pyproject.toml' found").  This script tries that command first and, when it
fails, does what such an install would have done for a flat package: it copies
the importable files unchanged -- the ``co_alibi_attn`` package and ``model.py``
-- into baseline/_ref, so that ``sys.path.insert(0, "baseline/_ref"); import
co_alibi_attn`` imports the reference exactly as its own scripts do
(co_alibi_attn/benchmark_flops.py adds the checkout root to sys.path).

Nothing under baseline/_ref is committed; it travels to the GPU box with the
working tree and is used only by baseline/triton_ref.py, the same-box comparator.
"""
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
DEST = os.path.join(HERE, "_ref")


def main():
    if len(sys.argv) != 2 or not os.path.isdir(os.path.join(sys.argv[1], "co_alibi_attn")):
        raise SystemExit("usage: python baseline/install_ref.py <reference checkout root holding co_alibi_attn/>")
    src = os.path.abspath(sys.argv[1])
    cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--find-links",
           "/opt/wheelhouse", "--target", DEST, src]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode == 0 and os.path.isdir(os.path.join(DEST, "co_alibi_attn")):
        how = "pip install --target"
    else:
        if os.path.isdir(DEST):
            shutil.rmtree(DEST)
        os.makedirs(DEST)
        shutil.copytree(os.path.join(src, "co_alibi_attn"), os.path.join(DEST, "co_alibi_attn"),
                        ignore=shutil.ignore_patterns("__pycache__"))
        shutil.copy2(os.path.join(src, "model.py"), os.path.join(DEST, "model.py"))
        last = (r.stderr.strip().splitlines() or ["(no output)"])[-1]
        how = f"copy of the package files (pip install failed: {last})"
    with open(os.path.join(DEST, "INSTALLED_BY.txt"), "w") as f:
        f.write(how + "\n")
    print(f"baseline/_ref: {how}")


if __name__ == "__main__":
    main()
