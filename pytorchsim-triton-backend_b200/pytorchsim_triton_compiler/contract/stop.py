"""Why a lowering stops on purpose (the reference's contract/stop.py:13-31): a Reason per decision, raised as
Refused, recorded by the process that compiled, and declared by a kernel file that expects it.

The B200 lowering adds its own reasons for tile programs it recognises but does not execute; it never falls
back to an approximate or CPU path."""
import dataclasses
import enum
import json
import os

RECORD = "00-stop.json"


class Reason(enum.Enum):
    # Reasons the reference's compiler states (kept so a kernel file's expect_stop still names one).
    TRITON_PASS_FAILED = "triton-pass-failed"
    ATOMICS = "atomics"
    DTYPE_NOT_RUN = "dtype-not-run"
    MATH_UNLOWERED = "math-unlowered"
    POINTER_BASE_UNTRACED = "pointer-base-untraced"
    FILL_VARIES = "fill-varies"
    POINTER_TILE_UNCONVERTED = "pointer-tile-unconverted"
    DESCRIPTOR_CANNOT_STATE = "descriptor-cannot-state"
    MATRIX_UNIT_ONE_ROW = "matrix-unit-one-row"
    MATRIX_UNIT_NO_FORMAT = "matrix-unit-no-format"
    SPAD_OVERFLOW = "spad-overflow"
    NOT_A_PREFETCH_CANDIDATE = "not-a-prefetch-candidate"
    RUNTIME_ATTRIBUTE = "runtime-attribute"
    TOG_MASK_START = "tog-mask-start"
    MASKED_STORE_NOT_A_BOX = "masked-store-not-a-box"
    MASKED_BOX_BEFORE_TENSOR = "masked-box-before-tensor"
    DIGIT_REFUSED = "digit-refused"
    # B200 lowering: the program's class is not one the executor runs, or a shape it does not run.
    PROGRAM_CLASS_UNKNOWN = "program-class-unknown"
    SHAPE_NOT_RUN = "shape-not-run"
    INDEX_NOT_AFFINE = "index-not-affine"


class Refusal(Exception):
    """A stop made on purpose; `reason` names the decision."""
    reason = None


class Refused(Refusal):
    def __init__(self, reason, message):
        super().__init__(message)
        self.reason = reason


def record(workdir, e):
    with open(os.path.join(workdir, RECORD), "w") as f:
        json.dump({"reason": e.reason.value, "message": str(e)}, f)


def recorded(workdir):
    path = os.path.join(workdir, RECORD)
    if not os.path.exists(path):
        return None
    with open(path) as f:
        got = json.load(f)
    return Reason(got["reason"]), got["message"]


def clear(workdir):
    try:
        os.unlink(os.path.join(workdir, RECORD))
    except FileNotFoundError:
        pass


@dataclasses.dataclass(frozen=True)
class Stop:
    """Where a refuse/blocked/open kernel stops: the step, and a Reason or a dotted exception name."""
    step: str
    reason: object

    def __post_init__(self):
        if not isinstance(self.reason, (Reason, str)):
            raise TypeError(f"Stop.reason is a Reason or a dotted exception name, not {self.reason!r}")
        if isinstance(self.reason, str) and "." not in self.reason:
            raise ValueError(f"Stop.reason {self.reason!r} is not a dotted exception name")
