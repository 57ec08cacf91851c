"""ASK external compiler worker for ask_b200 kernel artifacts.

The process interface of docs/en/compilers.md ("Process Interface"):

    python -m ask_b200.worker --probe --request request.json
    python -m ask_b200.worker --request request.json --output artifact.json

``--probe`` prints the dependency fingerprint ({"producer", "adapter_version"})
to stdout.  A compilation writes the artifact (external-kernel-artifact v2)
atomically -- a temporary file in the output's directory, then a rename -- and
exits 0; on failure it writes the diagnostic to stderr and exits 1, leaving
no output file.  See :mod:`ask_b200.artifact` for what a request may hold.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m ask_b200.worker", description=__doc__.splitlines()[0])
    ap.add_argument("--probe", action="store_true", help="print the dependency fingerprint and exit")
    ap.add_argument("--request", required=True, help="request JSON (protocol v2)")
    ap.add_argument("--output", help="where to write the artifact JSON")
    args = ap.parse_args(argv)
    try:
        with open(args.request) as f:
            request = json.load(f)
    except (OSError, json.JSONDecodeError) as e:
        print(f"ask_b200 worker: cannot read the request: {e}", file=sys.stderr)
        return 1
    from . import artifact  # loads the library only after the arguments are known to be sane
    if args.probe:
        print(json.dumps(artifact.probe(request)))
        return 0
    if not args.output:
        print("ask_b200 worker: --output is required to compile", file=sys.stderr)
        return 1
    try:
        result = artifact.build_artifact(request)
    except artifact.AskB200Error as e:
        print(f"ask_b200 worker: {e}", file=sys.stderr)
        return 1
    out_dir = os.path.dirname(os.path.abspath(args.output))
    fd, tmp = tempfile.mkstemp(prefix=".artifact-", suffix=".json", dir=out_dir)
    try:
        with os.fdopen(fd, "w") as f:
            json.dump(result, f)
        os.replace(tmp, args.output)
    except BaseException:
        if os.path.exists(tmp):
            os.unlink(tmp)
        raise
    return 0


if __name__ == "__main__":
    sys.exit(main())
