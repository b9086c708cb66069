"""failure.json: the record a stage that stopped leaves in its workdir, so the caller that chose the kernel
learns why without parsing logs.

The file's fields are those the reference's callers read ({"format": 1, "stage", "kind", "message"} plus
facts of the kind; pytorchsim_triton_compiler/contract/failure.py in the reference).  The kind comes from
the type of what stopped the stage: a Refused lowering is "refuse" (with its Reason under "reason"), a
failure the device or a kernel reported through the status word is "device" (its PTSIM_E_* value under
"code"), anything else is "error"."""
import dataclasses
import json
import os

FILE = "failure.json"
FORMAT = 1

REFUSED = "refuse"
DEVICE = "device"
ERROR = "error"
KINDS = (REFUSED, DEVICE, ERROR)


class FailureError(RuntimeError):
    """failure.json exists but cannot be read as this format."""


@dataclasses.dataclass(frozen=True)
class Failure:
    stage: str
    kind: str
    message: str
    facts: dict = dataclasses.field(default_factory=dict)

    def as_json(self):
        return {"format": FORMAT, "stage": self.stage, "kind": self.kind, "message": self.message, **self.facts}

    @classmethod
    def from_json(cls, got, where):
        if not isinstance(got, dict) or got.get("format") != FORMAT:
            raise FailureError(f"{where}: format {got.get('format') if isinstance(got, dict) else got!r}; "
                               f"this build reads format {FORMAT}")
        missing = [k for k in ("stage", "kind", "message") if k not in got]
        if missing:
            raise FailureError(f"{where}: no {', '.join(missing)}")
        facts = {k: v for k, v in got.items() if k not in ("format", "stage", "kind", "message")}
        return cls(got["stage"], got["kind"], got["message"], facts)


def _path(workdir):
    return os.path.join(workdir, FILE)


def leave(workdir, stage, kind, message, **facts):
    """Write the record of a stage that stopped; returns its path."""
    if kind not in KINDS:
        raise ValueError(f"failure kind {kind!r} is not one of {KINDS}")
    rec = Failure(stage, kind, message, facts)
    with open(_path(workdir), "w") as fh:
        fh.write(json.dumps(rec.as_json(), indent=2) + "\n")
    return _path(workdir)


def found(workdir):
    """The Failure left in `workdir`, or None when the run there stopped nowhere."""
    try:
        with open(_path(workdir)) as fh:
            text = fh.read()
    except FileNotFoundError:
        return None
    try:
        got = json.loads(text)
    except json.JSONDecodeError as e:
        raise FailureError(f"{_path(workdir)}: not JSON ({e})") from None
    return Failure.from_json(got, _path(workdir))


def forget(workdir):
    """Drop the record an earlier run left, before a new run can stop."""
    if os.path.exists(_path(workdir)):
        os.remove(_path(workdir))
