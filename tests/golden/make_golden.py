"""Copy the reference's SHA-256 pins into tests/golden/.

The reference commits the SHA-256 of every input, output and graph file that
ref/build.sh writes, for both ggml builds (evidence/ref-stock.sha256 and
evidence/ref-pinned.sha256). These are the golden vectors the oracle and the
CUDA path are checked against. Run once in a container that has the reference:

    python tests/golden/make_golden.py <reference-root>
"""
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def main(ref_root: str) -> None:
    for flavour in ("stock", "pinned"):
        src = os.path.join(ref_root, "evidence", "ref-%s.sha256" % flavour)
        with open(src) as f:
            lines = [ln.rstrip("\n") for ln in f if ln.strip()]
        dst = os.path.join(HERE, "ref-%s.sha256" % flavour)
        with open(dst, "w") as f:
            f.write("\n".join(lines) + "\n")
        print("wrote", dst, len(lines), "hashes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <reference-root>")
    main(sys.argv[1])
