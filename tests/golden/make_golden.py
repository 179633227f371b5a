"""Extracts the routing / RMSNorm / expert / Hyper-Connection sections of the reference's operator fixture into
tests/golden/deepseek_v4_operators.json (run in a container that has the reference tree).

Source: tests/fixtures/deepseek_v4_operators.json of the vastloom reference ("pure-Python
translation of pinned model.py/kernel.py equations"), consumed there by
test_deepseek_v4_reference_operators (tests/test_main.cpp:4330) with absolute tolerance 3e-5.

    python tests/golden/make_golden.py [/path/to/reference]
"""
import json
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[2]))
from vastloom_b200.build import reference_root  # noqa: E402

ref = Path(sys.argv[1]) if len(sys.argv) > 1 else reference_root()
src = json.loads((ref / "tests" / "fixtures" / "deepseek_v4_operators.json").read_text())
keep = {k: src[k] for k in ("learned_route", "hash_route", "rms_norm", "expert", "hyper_connection", "absolute_tolerance",
                            "official_revision")}
out = Path(__file__).resolve().parent / "deepseek_v4_operators.json"
out.write_text(json.dumps(keep, indent=1, sort_keys=True) + "\n")
print(f"wrote {out}")
