"""Writes tests/golden/stagewire_frames.jsonl: Stagewire v2 frames made by the
reference runtime's own C++ encoder (runtime/protocol/stage.cpp, through the
`golden` mode of oracle/_ref/transport_replay), each with what the reference's
request decoder reads back from it (`decode` mode; response frames carry no
decoder record). Run where the reference tree is present:

    python tests/golden/make_stagewire_frames.py
"""
from __future__ import annotations

import importlib.util
import json
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent


def main() -> None:
    spec = importlib.util.spec_from_file_location("jfb_ref_transport_build",
                                                  REPO / "oracle" / "ref_transport" / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    binary = mod.build()
    if binary is None:
        raise SystemExit("the reference tree is needed to make these frames")
    lines = subprocess.run([str(binary), "golden"], capture_output=True, text=True, check=True).stdout.splitlines()
    frames = [json.loads(l) for l in lines if l.strip()]
    requests = [f for f in frames if not f["name"].startswith("response")]
    decoded = subprocess.run([str(binary), "decode"], input="\n".join(f["frame"] for f in requests) + "\n",
                             capture_output=True, text=True, check=True).stdout.splitlines()
    for f, d in zip(requests, decoded):
        f["reference_decode"] = json.loads(d)
    with open(HERE / "stagewire_frames.jsonl", "w") as out:
        for f in frames:
            out.write(json.dumps(f) + "\n")
    print(f"wrote {len(frames)} frames")


if __name__ == "__main__":
    main()
