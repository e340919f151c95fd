"""Copy the reference's conformance vectors that pin the HardShell path into tests/golden/.

Run once in a container that has the reference checkout (its path is the first argument):

    python tests/golden/make_fixtures.py <reference checkout>

The files are the reference's own golden data (conformance/README.md of the reference):
the tiny model `tiny.hsm`, the version 2 container vectors of the `text` profile, with
`vectors.tsv`, and the version 1 container `taco-v1-tiny.taco` (folded with another tiny model,
the one of the reference's Rust test builder: it pins the reading of a version 1 header). The profile `logs` and `auto` vectors (mixed blocks) are not copied: the mixer
is outside the path this backend serves. The script writes MANIFEST.tsv with the SHA-256 of
every copied file, so a test can check that the fixtures are the published bytes.
"""

import hashlib
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
TEXT_VECTORS = [
    "empty", "one_byte", "random_raw", "text_k0", "text_k20", "text_kinds",
    "predicted_text_k0", "predicted_text_k32", "all_kinds_text",
]


def main() -> int:
    ref = Path(sys.argv[1])
    conf = ref / "conformance"
    files = [("tiny.hsm", conf / "tiny.hsm"), ("vectors.tsv", conf / "v2" / "vectors.tsv"),
             ("taco_v1_tiny.taco", conf / "taco-v1-tiny.taco")]
    for name in TEXT_VECTORS:
        for ext in (".in", ".taco"):
            files.append((name + ext, conf / "v2" / (name + ext)))
    lines = []
    for dst, src in files:
        shutil.copyfile(src, HERE / dst)
        lines.append(f"{dst}\t{hashlib.sha256(src.read_bytes()).hexdigest()}")
    (HERE / "MANIFEST.tsv").write_text("\n".join(lines) + "\n")
    print(f"copied {len(files)} files into {HERE}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
