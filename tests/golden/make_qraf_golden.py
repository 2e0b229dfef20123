"""Write the .qraf golden file with the reference's OWN writer.

Run where the reference tree exists (it builds oracle/_ref first):

    python tests/golden/make_qraf_golden.py

Output (committed): llama_like_ref.qraf — tests/qraf_spec.py's llama_like()
model written by the reference's QrafWriter (src/qraf/writer.cpp:83-308) with
tensors quantized by the reference's quantize_q8_0 / quantize_q4_0
(src/tensor/quantize.cpp:105-183).  The writer test rebuilds the same model with
qraf_b200.qraf_file.QrafFileWriter and compares the files byte for byte.
"""
from __future__ import annotations

import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(HERE))

import oracle  # noqa: E402
import qraf_spec  # noqa: E402

OUT = os.path.join(HERE, "llama_like_ref.qraf")


def main() -> None:
    oracle.build(with_ref=True)
    ref = oracle.Reference()
    spec = qraf_spec.llama_like()
    ref.write_qraf(OUT, **qraf_spec.reference_args(spec, ref.quantize_rows))
    print(OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main()
