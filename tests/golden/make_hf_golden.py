"""Copies the reference's Hugging Face test fixtures into tests/golden/hf/.

The Kotensor test suite holds three tiny checkpoints with the logits Hugging
Face computed for them (src/test/resources/hf/{llama_tiny, llama3_tiny,
qwen_tiny_sharded}: config.json, the safetensors weights, expected.json with
input ids and per-position logits) and a dtype fixture (hf/dtypes).  These are
the reference's own known answers for the decode path (HuggingFaceImportTest
checks its decoder against them at 2e-4) and for the safetensors conversion.
The files are copied unchanged (data, not code) so the tests that pin the
oracle to them do not depend on the reference tree being present; nothing
else is copied (tokenizer.json is not used).

Run: python tests/golden/make_hf_golden.py <Kotensor project directory>
     (the directory holding src/test/resources/hf)
"""
from __future__ import annotations

import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
FIXTURES = {
    "llama_tiny": ["config.json", "expected.json", "model.safetensors"],
    "llama3_tiny": ["config.json", "expected.json", "model.safetensors"],
    "qwen_tiny_sharded": ["config.json", "expected.json", "model.safetensors.index.json",
                          "model-00001-of-00002.safetensors", "model-00002-of-00002.safetensors"],
    "dtypes": ["dtypes.safetensors", "expected.json"],
}


def main(project: str) -> None:
    src_root = os.path.join(project, "src", "test", "resources", "hf")
    if not os.path.isdir(src_root):
        raise SystemExit(f"no src/test/resources/hf under {project}")
    for name, files in FIXTURES.items():
        dst = os.path.join(HERE, "hf", name)
        os.makedirs(dst, exist_ok=True)
        for f in files:
            shutil.copyfile(os.path.join(src_root, name, f), os.path.join(dst, f))
            print(os.path.join("tests", "golden", "hf", name, f))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit(__doc__)
    main(sys.argv[1])
