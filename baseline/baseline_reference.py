"""Reference arm of bench.py: the unmodified reference (installed into baseline/_ref) on the same metric/config.

Prints one JSON line with "impl": "reference".  Until the harness that drives
the reference's own trainer on the synthetic OLMoE-shaped configuration is in
place, it reports the arm as unavailable with the reason.
"""

from __future__ import annotations

import json
import os

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(HERE, "_ref")


def main(args) -> int:
    if not os.path.isdir(os.path.join(REF, "veomni")):
        print(json.dumps({"impl": "reference", "unavailable": "reference not installed in baseline/_ref"}))
        return 0
    print(json.dumps({"impl": "reference",
                      "unavailable": "reference harness for the OLMoE-shaped synthetic run is not implemented yet"}))
    return 0
