"""Install the unmodified reference into baseline/_ref (git-ignored) for
``bench.py --impl reference``.

    python baseline/install_reference.py [REFERENCE_CHECKOUT]

First tries the offline pip install the benchmark contract names
(``pip install --no-index --no-build-isolation --find-links /opt/wheelhouse
--target baseline/_ref <checkout>``).  The reference builds with hatchling,
which the offline wheelhouse does not carry, so that step fails here; the
fallback then places the package tree exactly as its wheel would
(``[tool.hatch.build.targets.wheel] packages = ["src/nano_inference"]``):
``<checkout>/src/nano_inference`` -> ``baseline/_ref/nano_inference``,
byte for byte.  The benchmark imports only ``nano_inference.sampling`` and
``nano_inference.core.sampling`` from it (torch and dataclasses).
"""
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
TARGET = os.path.join(HERE, "_ref")


def main():
    src = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("NANO_INFERENCE_REFERENCE", "")
    if not src or not os.path.isdir(src):
        sys.exit("usage: install_reference.py REFERENCE_CHECKOUT")
    r = subprocess.run([sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation",
                        "--find-links", "/opt/wheelhouse", "--no-deps", "--target", TARGET, src],
                       capture_output=True, text=True)
    if r.returncode == 0:
        print("pip install: ok")
        return
    print("pip install failed:", (r.stderr.strip().splitlines() or ["?"])[-1])
    pkg = os.path.join(src, "src", "nano_inference")
    dst = os.path.join(TARGET, "nano_inference")
    if os.path.isdir(dst):
        shutil.rmtree(dst)
    shutil.copytree(pkg, dst, ignore=shutil.ignore_patterns("__pycache__"))
    with open(os.path.join(TARGET, "INSTALLED_FROM"), "w") as f:
        f.write(f"package tree of {src} (pip failed: {(r.stderr.strip().splitlines() or ['?'])[-1]})\n")
    print("copied package tree ->", dst)


if __name__ == "__main__":
    main()
