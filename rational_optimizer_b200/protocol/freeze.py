"""Source freeze: SHA-256 inventory of a repository's public sources (behaviour of
experiments/protocol/build_source_freeze.py:1-199; same ``sha256sum`` line
format, ``<hex>  <relative path>``, sorted by path).

The inventory is what a clean clone exposes: ``git ls-files --cached
--others --exclude-standard``, regular files only (no symlinks).  Sources are
selected by suffix or name; generated artefacts (binaries, checkpoints,
images, caches, results, logs) never are.  :func:`check` reports the
difference between a committed freeze and the working tree as
added / removed / changed paths instead of a bare pass/fail.

    python -m rational_optimizer_b200.protocol.freeze [--root .] [--output SOURCE_FREEZE.sha256] [--check]
"""
from __future__ import annotations

import argparse
import hashlib
import os
import subprocess
import tempfile
from dataclasses import dataclass
from pathlib import Path

SOURCE_SUFFIXES = frozenset({".c", ".cc", ".cpp", ".cu", ".cuh", ".h", ".hpp", ".py", ".pyi", ".sbatch", ".sh",
                             ".toml", ".yaml", ".yml"})
SOURCE_NAMES = frozenset({"pytest.ini", "requirements.txt", "setup.py"})
ARTEFACT_SUFFIXES = frozenset({".bin", ".ckpt", ".dll", ".dylib", ".egg", ".gif", ".jpeg", ".jpg", ".npy", ".npz",
                               ".o", ".pdf", ".png", ".pt", ".pth", ".pyc", ".so", ".tar", ".tgz", ".whl", ".zip"})
EXCLUDED_DIRS = ("experiments/cache/", "experiments/failed_attempts/", "experiments/logs/", "experiments/results/",
                 "experiments/runs/")


class FreezeError(RuntimeError):
    pass


def public_files(root) -> list[str]:
    root = Path(root)
    try:
        out = subprocess.run(["git", "-C", str(root), "ls-files", "--cached", "--others", "--exclude-standard"],
                             check=True, capture_output=True, text=True).stdout
    except (FileNotFoundError, subprocess.CalledProcessError) as exc:
        raise FreezeError(f"{root} is not a git work tree") from exc
    files = {Path(rel).as_posix() for rel in out.splitlines()}
    return sorted(rel for rel in files if (root / rel).is_file() and not (root / rel).is_symlink())


def is_source(rel: str, *, manifests=frozenset(), output: str | None = None) -> bool:
    p = Path(rel)
    if rel == output or rel.startswith(EXCLUDED_DIRS) or "__pycache__" in p.parts:
        return False
    suffix = p.suffix.lower()
    if suffix in ARTEFACT_SUFFIXES:
        return False
    return rel in manifests or p.name in SOURCE_NAMES or suffix in SOURCE_SUFFIXES


@dataclass
class Freeze:
    root: Path
    entries: dict  # relative path -> sha256

    @classmethod
    def collect(cls, root, *, manifests=(), required=(), output=None):
        """Hash the public sources under ``root``; ``manifests`` (non-source files to
        include) and ``required`` paths must all be present."""
        root = Path(root)
        manifests = frozenset(manifests)
        chosen = [rel for rel in public_files(root) if is_source(rel, manifests=manifests, output=output)]
        missing = sorted((manifests | frozenset(required)) - set(chosen))
        if missing:
            raise FreezeError(f"required files are not public sources: {', '.join(missing)}")
        entries = {rel: hashlib.sha256((root / rel).read_bytes()).hexdigest() for rel in chosen}
        return cls(root, entries)

    def render(self) -> str:
        return "".join(f"{h}  {rel}\n" for rel, h in sorted(self.entries.items()))

    @staticmethod
    def parse(text: str) -> dict:
        out = {}
        for n, line in enumerate(text.splitlines(), 1):
            digest, sep, rel = line.partition("  ")
            if not sep or len(digest) != 64 or any(c not in "0123456789abcdef" for c in digest) or not rel:
                raise FreezeError(f"line {n} is not '<sha256>  <path>': {line!r}")
            if rel in out:
                raise FreezeError(f"line {n} repeats {rel}")
            out[rel] = digest
        return out

    def write(self, path) -> None:
        path = Path(path)
        path.parent.mkdir(parents=True, exist_ok=True)
        fd, tmp = tempfile.mkstemp(prefix=f".{path.name}.", dir=path.parent, text=True)
        try:
            with os.fdopen(fd, "w", encoding="utf-8", newline="") as fh:
                fh.write(self.render())
            os.replace(tmp, path)
        finally:
            Path(tmp).unlink(missing_ok=True)

    def diff(self, frozen: dict) -> dict:
        """{"added": [...], "removed": [...], "changed": [...]} of the tree against ``frozen``."""
        return {"added": sorted(set(self.entries) - set(frozen)),
                "removed": sorted(set(frozen) - set(self.entries)),
                "changed": sorted(rel for rel in set(self.entries) & set(frozen) if self.entries[rel] != frozen[rel])}


def check(path, root, **kw) -> dict:
    """Differences between the freeze file at ``path`` and the tree (empty lists: up to date)."""
    path = Path(path)
    if not path.is_file():
        raise FreezeError(f"no source freeze at {path}")
    output = path.resolve().relative_to(Path(root).resolve()).as_posix() if path.resolve().is_relative_to(
        Path(root).resolve()) else None
    tree = Freeze.collect(root, output=output, **kw)
    return tree.diff(Freeze.parse(path.read_text(encoding="utf-8")))


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--root", type=Path, default=Path("."))
    ap.add_argument("--output", type=Path, default=Path("SOURCE_FREEZE.sha256"))
    ap.add_argument("--check", action="store_true", help="compare with the existing freeze, write nothing")
    a = ap.parse_args(argv)
    out = a.output if a.output.is_absolute() else a.root / a.output
    try:
        if a.check:
            d = check(out, a.root)
            if any(d.values()):
                print(f"FAIL source freeze is stale: {d}")
                return 1
            print(f"PASS source freeze ({len(Freeze.parse(out.read_text()))} files)")
            return 0
        rel = out.resolve().relative_to(a.root.resolve()).as_posix()
        freeze = Freeze.collect(a.root, output=rel)
        freeze.write(out)
        print(f"wrote {out} ({len(freeze.entries)} files)")
        return 0
    except FreezeError as exc:
        print(f"FAIL {exc}")
        return 1


if __name__ == "__main__":
    raise SystemExit(main())
