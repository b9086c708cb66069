"""Deliberate stops of the lowering.

A program the B200 executor does not run is refused, never approximated: the lowering raises `Refused`
with a `Reason`, the compile stage leaves failure.json of kind "refuse" naming the Reason's value, and a
kernel file that expects the stop declares where and why with `Stop(step, reason)` in its KernelSpec.

The Reason values are the reference's (pytorchsim_triton_compiler/contract/stop.py:13-31), so a kernel file
written for the reference still names its stop; the last three are this executor's own."""
import enum


class Reason(enum.Enum):
    # Decisions of the reference's MLIR lowering, kept as names a kernel file may declare.
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
    # The B200 lowering: no executor class matches the program, the class does not run this shape, or an
    # index is not an affine digit expression of the program's variables.
    PROGRAM_CLASS_UNKNOWN = "program-class-unknown"
    SHAPE_NOT_RUN = "shape-not-run"
    INDEX_NOT_AFFINE = "index-not-affine"


class Refused(Exception):
    """The lowering declines a program on purpose.  `reason` is the Reason; str(e) says what was seen."""

    def __init__(self, reason, message):
        if not isinstance(reason, Reason):
            raise TypeError(f"a refusal names a Reason, got {reason!r}")
        super().__init__(message)
        self.reason = reason


def _valid_reason(reason):
    """A Reason, or the dotted name of the Python exception an open kernel dies on ("pkg.Error")."""
    if isinstance(reason, Reason):
        return reason
    if not isinstance(reason, str):
        raise TypeError(f"a Stop's reason is a Reason or a dotted exception name, not {reason!r}")
    owner, _, leaf = reason.rpartition(".")
    if not owner or not leaf.isidentifier():
        raise ValueError(f"{reason!r} is not a dotted exception name (module.Exception)")
    return reason


class Stop:
    """Where a kernel that is not expected to pass stops: the stage (`step`) and the Reason (or, for an open
    kernel, the dotted exception name).  Immutable and comparable, so a test can compare it with what the
    compile recorded."""
    __slots__ = ("step", "reason")

    def __init__(self, step, reason):
        object.__setattr__(self, "step", str(step))
        object.__setattr__(self, "reason", _valid_reason(reason))

    def __setattr__(self, name, value):
        raise AttributeError("a Stop does not change once declared")

    def __eq__(self, other):
        return isinstance(other, Stop) and (self.step, self.reason) == (other.step, other.reason)

    def __hash__(self):
        return hash((self.step, self.reason))

    def __repr__(self):
        return f"Stop({self.step!r}, {self.reason!r})"
