"""Regenerate the golden fixtures in this folder from the reference sources
(run in a checkout that has the reference tree; the fixtures are committed so
the tests never read it).

* focrq_minimal_header.json -- the "Minimal Header Example" JSON of the
  reference's `.focrq` format document (docs/focrq-format.md).
* model_registry.json -- every `id` / `license_notice` pair of the reference's
  architecture registry (src/native_engine/model_arch.rs) plus the default
  model notice (src/lib.rs FOCR_MODEL_LICENSE_NOTICE).

Usage: python tests/golden/make_golden.py <reference checkout>
"""
import json
import re
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def main(ref: Path) -> None:
    doc = (ref / "docs" / "focrq-format.md").read_text()
    sec = doc[doc.index("## Minimal Header Example"):]
    body = sec[sec.index("```json") + len("```json"):]
    header = json.loads(body[:body.index("```")])
    (HERE / "focrq_minimal_header.json").write_text(json.dumps(header, indent=1, sort_keys=True) + "\n")

    arch = (ref / "src" / "native_engine" / "model_arch.rs").read_text()
    lib = (ref / "src" / "lib.rs").read_text()
    notice = re.search(r'FOCR_MODEL_LICENSE_NOTICE: &str =\s*"([^"]+)"', lib).group(1)
    reg = {"unlimited-ocr": notice}
    for m in re.finditer(r'id:\s*"([^"]+)",\s*display_name:[^\n]*\n\s*license_notice:\s*"([^"]+)"', arch):
        reg[m.group(1)] = m.group(2)
    (HERE / "model_registry.json").write_text(json.dumps(reg, indent=1, sort_keys=True) + "\n")


if __name__ == "__main__":
    main(Path(sys.argv[1]))
