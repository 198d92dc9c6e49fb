"""Recipe: an unmodified copy of the reference's Python package under
baseline/_ref (git-ignored; it travels with the working tree to the GPU box),
for the benchmark's reference arms only: the reference's own CPU path
(gsp.runtime.constrained_projection on CPU tensors) and its own Triton kernels
(gsp.triton_runtime) timed on the same GPU. The reference has no setup.py or
pyproject, so the package directory is copied byte for byte; SOURCE.json
records each file's sha256.

usage: python baseline/install_reference.py /path/to/reference/checkout
"""
import hashlib
import json
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def main(src_root: str) -> None:
    src = os.path.join(src_root, "gsp")
    if not os.path.isdir(src):
        raise SystemExit(f"{src} is not the reference's gsp package")
    dst_root = os.path.join(HERE, "_ref")
    dst = os.path.join(dst_root, "gsp")
    if os.path.exists(dst_root):
        shutil.rmtree(dst_root)
    os.makedirs(dst)
    files = {}
    for name in sorted(os.listdir(src)):
        if name.endswith(".py"):
            shutil.copyfile(os.path.join(src, name), os.path.join(dst, name))
            with open(os.path.join(dst, name), "rb") as f:
                files[name] = hashlib.sha256(f.read()).hexdigest()
    with open(os.path.join(dst_root, "SOURCE.json"), "w") as f:
        json.dump({"package": "gsp", "files": files}, f, indent=1)
    print(f"copied {len(files)} files into {dst}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit(__doc__)
    main(sys.argv[1])
