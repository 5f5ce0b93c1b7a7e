"""Installs the unmodified reference tokenserve package into ``baseline/_ref``.

``pip install --no-index --no-build-isolation --target baseline/_ref <reference>`` cannot build
the reference here: its build backend (hatchling, ``pyproject.toml`` ``[build-system]``) is not
in the offline wheelhouse. tokenserve is pure Python and its wheel target is just the
``src/tokenserve`` package (``[tool.hatch.build.targets.wheel] packages``), so this script
writes that wheel itself — the package's files byte for byte, plus the metadata
(``METADATA``, ``WHEEL``, ``entry_points.txt``, ``RECORD``) from ``pyproject.toml`` — and
installs it with pip (``--no-index --no-deps``: fastapi, uvicorn, pydantic and
prometheus-client are already in the image).

``baseline/_ref`` is kept out of git and travels with the tree to the GPU box, where the tests
that drive tokenserve's own ``Engine`` and the bench's reference arm import it.

    python baseline/install_reference.py [path/to/tokenserve]
"""

from __future__ import annotations

import base64
import hashlib
import os
import subprocess
import sys
import tempfile
import tomllib
import zipfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
TARGET = HERE / "_ref"


def _record_hash(data: bytes) -> str:
    digest = base64.urlsafe_b64encode(hashlib.sha256(data).digest()).rstrip(b"=").decode()
    return f"sha256={digest}"


def build_wheel(repo: Path, out_dir: Path) -> Path:
    meta = tomllib.loads((repo / "pyproject.toml").read_text())["project"]
    name, version = meta["name"], meta["version"]
    pkg_dirs = tomllib.loads((repo / "pyproject.toml").read_text())["tool"]["hatch"]["build"][
        "targets"]["wheel"]["packages"]  # fmt: skip
    files: list[tuple[str, bytes]] = []
    for pkg in pkg_dirs:
        root = repo / pkg
        for p in sorted(root.rglob("*")):
            if p.is_dir() or "__pycache__" in p.parts or p.suffix == ".pyc":
                continue
            files.append((f"{root.name}/{p.relative_to(root).as_posix()}", p.read_bytes()))
    dist = f"{name}-{version}.dist-info"
    lines = ["Metadata-Version: 2.1", f"Name: {name}", f"Version: {version}"]
    if "description" in meta:
        lines.append(f"Summary: {meta['description']}")
    if "requires-python" in meta:
        lines.append(f"Requires-Python: {meta['requires-python']}")
    lines += [f"Requires-Dist: {d}" for d in meta.get("dependencies", [])]
    files.append((f"{dist}/METADATA", ("\n".join(lines) + "\n").encode()))
    files.append((f"{dist}/WHEEL", b"Wheel-Version: 1.0\nGenerator: install_reference\n"
                                   b"Root-Is-Purelib: true\nTag: py3-none-any\n"))  # fmt: skip
    scripts = meta.get("scripts", {})
    if scripts:
        ep = "[console_scripts]\n" + "".join(f"{k} = {v}\n" for k, v in scripts.items())
        files.append((f"{dist}/entry_points.txt", ep.encode()))
    record = "".join(f"{n},{_record_hash(d)},{len(d)}\n" for n, d in files) + f"{dist}/RECORD,,\n"
    files.append((f"{dist}/RECORD", record.encode()))
    wheel = out_dir / f"{name}-{version}-py3-none-any.whl"
    with zipfile.ZipFile(wheel, "w", zipfile.ZIP_DEFLATED) as z:
        for n, d in files:
            z.writestr(n, d)
    return wheel


def default_repo() -> Path | None:
    """Where the reference lives in the build container, if it is there."""
    src = os.environ.get("TOKENSERVE_REPO") or "/root/reference"
    return Path(src) if (Path(src) / "pyproject.toml").exists() else None


def installed() -> bool:
    return (TARGET / "tokenserve" / "engine.py").exists()


def install(repo: Path) -> Path:
    with tempfile.TemporaryDirectory() as tmp:
        wheel = build_wheel(repo, Path(tmp))
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-deps", "--upgrade",
               "--target", str(TARGET), str(wheel)]  # fmt: skip
        subprocess.run(cmd, check=True, capture_output=True, text=True)
    return TARGET


if __name__ == "__main__":
    repo = Path(sys.argv[1]) if len(sys.argv) > 1 else default_repo()
    if repo is None:
        sys.exit("install_reference.py: give the tokenserve repository (or set TOKENSERVE_REPO)")
    print(install(repo))
