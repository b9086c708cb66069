"""failure.json, the record a stopped compile or launch leaves in its workdir (the reference's
contract/failure.py:1-63): written from the type of what stopped, never from what it printed."""
import json
import os

FILE = "failure.json"
FORMAT = 1

SPAD_OVERFLOW = "spad-overflow"
NOT_A_PREFETCH_CANDIDATE = "not-a-prefetch-candidate"
SPILL_NOT_ALLOWED = "spill-not-allowed"
REFUSED = "refuse"
ERROR = "error"
DEVICE = "device"
"""The executor (or a kernel, through the status word) reported a failure: "code" holds the PTSIM_E_* value."""


class FailureError(RuntimeError):
    pass


def clear(workdir):
    try:
        os.unlink(os.path.join(workdir, FILE))
    except FileNotFoundError:
        pass


def write(workdir, stage, kind, message, **facts):
    with open(os.path.join(workdir, FILE), "w") as fh:
        json.dump({"format": FORMAT, "stage": stage, "kind": kind, "message": message, **facts}, fh, indent=2)
        fh.write("\n")


def read(workdir):
    path = os.path.join(workdir, FILE)
    try:
        with open(path) as fh:
            got = json.load(fh)
    except FileNotFoundError:
        return None
    except json.JSONDecodeError as e:
        raise FailureError(f"{path}: not valid JSON ({e})")
    if got.get("format") != FORMAT:
        raise FailureError(f"{path}: format {got.get('format')!r}, this build reads format {FORMAT}")
    return got
