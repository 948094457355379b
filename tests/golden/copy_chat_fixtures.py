"""Copies the reference's chat fixtures used by tests/test_chat.py into tests/golden/:
fixtures/m12_chatml_corpus.json (ChatML cases with expected prompts and rejections, made by
the reference's tools/oracle/oracle_chatml.py from the upstream template) and the small BPE
tokenizer directory fixtures/m12_tokenizer/ (tokenizer.json, tokenizer_config.json,
generation_config.json, config.json).  Run once where a reference checkout exists:

    python tests/golden/copy_chat_fixtures.py /path/to/reference
"""
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def main(ref: str):
    shutil.copyfile(os.path.join(ref, "fixtures", "m12_chatml_corpus.json"),
                    os.path.join(HERE, "m12_chatml_corpus.json"))
    os.makedirs(os.path.join(HERE, "m12_tokenizer"), exist_ok=True)
    for f in ("tokenizer.json", "tokenizer_config.json", "generation_config.json", "config.json"):
        shutil.copyfile(os.path.join(ref, "fixtures", "m12_tokenizer", f), os.path.join(HERE, "m12_tokenizer", f))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: copy_chat_fixtures.py <reference checkout>")
    main(sys.argv[1])
