"""Install the unmodified nano-vLLM reference into baseline/_ref.

The drop-in tests (install() into the reference's Qwen3Attention and
ModelRunner, decode metadata against its prepare_decode, the row-parallel
dispatch), the engine workload of bench.py and the reference's own modules
used as comparison paths all import nano-vLLM from baseline/_ref.  This step
installs it there, offline and without dependencies (they are in the image):

    python -m pip install --no-index --no-build-isolation --no-deps --target baseline/_ref <copy>

from a temporary copy of the checkout, because the build writes into its
source tree.  The checkout's directory comes from argv[1], else the
NANOVLLM_REF environment variable, else the development container's default
location.  Without a checkout (a GPU box receives baseline/_ref ready-made
with the rest of the repository) nothing is done.  An existing install whose
recorded source hash matches the checkout is kept.

    python baseline/install_reference.py [checkout]
"""
import hashlib
import os
import shutil
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
TARGET = os.path.join(HERE, "_ref")
STAMP = os.path.join(TARGET, ".source_sha256")
DEFAULT_CHECKOUT = "/root/reference"


def checkout_dir(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    if argv:
        return argv[0]
    return os.environ.get("NANOVLLM_REF") or DEFAULT_CHECKOUT


def source_hash(src):
    """SHA-256 over the package sources and pyproject of a checkout (sorted paths)."""
    h = hashlib.sha256()
    files = [os.path.join(src, "pyproject.toml")]
    for root, _, names in os.walk(os.path.join(src, "nanovllm")):
        files += [os.path.join(root, n) for n in names if n.endswith(".py")]
    for f in sorted(files):
        h.update(os.path.relpath(f, src).encode())
        with open(f, "rb") as fh:
            h.update(fh.read())
    return h.hexdigest()


def installed():
    return os.path.isdir(os.path.join(TARGET, "nanovllm"))


def install(src=None, quiet=True):
    """Install the checkout into baseline/_ref; returns the target, or None when
    there is no checkout to install from (the install already present, if any, stays)."""
    src = src or checkout_dir([])
    if not os.path.isfile(os.path.join(src, "pyproject.toml")):
        return TARGET if installed() else None
    want = source_hash(src)
    if installed() and os.path.exists(STAMP):
        with open(STAMP) as fh:
            if fh.read().strip() == want:
                return TARGET
    with tempfile.TemporaryDirectory(prefix="nanovllm_src_") as tmp:
        copy = os.path.join(tmp, "src")
        shutil.copytree(src, copy, ignore=shutil.ignore_patterns(".git", "__pycache__", "*.egg-info", "build"))
        if os.path.isdir(TARGET):
            shutil.rmtree(TARGET)
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
               "--target", TARGET, copy]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"installing the reference failed:\n{r.stdout}\n{r.stderr}")
    with open(STAMP, "w") as fh:
        fh.write(want + "\n")
    if not quiet:
        print(f"nano-vLLM installed into {TARGET}")
    return TARGET


if __name__ == "__main__":
    where = install(checkout_dir(), quiet=False)
    if where is None:
        sys.exit("no reference checkout found (pass its directory or set NANOVLLM_REF)")
