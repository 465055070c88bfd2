"""Copy the reference's own golden fixtures for the encoder path into
tests/golden/, so that the parity tests run where the reference tree is absent.

    python tests/golden/make_golden.py REFERENCE_ROOT

REFERENCE_ROOT is the root of a checkout of the reference repository.

Copied as-is (no regeneration): each fixture is a tiny random Hugging Face
checkpoint plus the golden outputs the reference's tests assert against.
  * tiny_splade            crates/inl-sparse/tests/fixtures/tiny_splade/
                           (ModernBERT MLM + ShiftedTopKSpladePooling; asserted by
                           crates/inl-sparse/src/modernbert.rs:1034-1057, |dw| <= 1e-4,
                           identical term sets). Directory layout kept, as
                           the loader follows modules.json.
  * tiny_embeddinggemma2   crates/inl-text/tests/fixtures/tiny_embeddinggemma2/
                           (EmbeddingGemma 2 text tower; asserted by
                           crates/inl-text/src/gemma2.rs:941-967, |d| < 2e-5)
  * tiny_qwen3_5_late      crates/inl-late/tests/fixtures/tiny_qwen3_5_late/
                           (Qwen3.5 tower with Gated DeltaNet and gated full
                           attention, 1_Dense, the document skiplist;
                           asserted by crates/inl-late/tests/tiny_golden.rs,
                           max |d| < 1e-4: pins oracle/qwen3_5.py and the
                           host's task handling). Directory layout kept, as
                           the loader follows modules.json.
"""
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
FIXTURES = {
    "tiny_splade": ("crates/inl-sparse/tests/fixtures/tiny_splade",
                    ["config.json", "model.safetensors", "golden.json", "1_ShiftedTopKSpladePooling/config.json",
                     "tokenizer.json", "modules.json", "config_sentence_transformers.json"]),
    "tiny_embeddinggemma2": ("crates/inl-text/tests/fixtures/tiny_embeddinggemma2",
                             ["config.json", "model.safetensors", "golden.json", "tokenizer.json"]),
    "tiny_qwen3_5_late": ("crates/inl-late/tests/fixtures/tiny_qwen3_5_late",
                          ["config.json", "config_sentence_transformers.json", "sentence_bert_config.json",
                           "modules.json", "2_MultiVectorMask/config.json", "tokenizer.json", "golden.json",
                           "model.safetensors", "1_Dense/config.json", "1_Dense/model.safetensors",
                           "3_Normalize/config.json"]),
}
KEEP_DIRS = {"tiny_qwen3_5_late", "tiny_splade"}


def main(ref_root: str) -> None:
    ref = Path(ref_root)
    for name, (rel, files) in FIXTURES.items():
        for f in files:
            src = ref / rel / f
            dst = HERE / name / (f if name in KEEP_DIRS else f.replace("/", "__"))
            dst.parent.mkdir(parents=True, exist_ok=True)
            shutil.copyfile(src, dst)
            print(f"{src} -> {dst.relative_to(HERE)}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py REFERENCE_ROOT")
    main(sys.argv[1])
