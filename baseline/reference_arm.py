"""Reference arm of ``bench.py``: the reference engine, unmodified, on the same workload.

Placeholder until the reference's stock path is wired up: prints the ``unavailable`` line.
"""

from __future__ import annotations

import json
import os


def main(args, report) -> None:
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps({"impl": "reference", "unavailable": "reference arm not wired yet"}), flush=True)
