"""The Triton backend plugin, compile side, kept call-compatible with the reference
(pytorchsim_triton_compiler/triton_extension/python/pytorchsim_triton_backend/compiler.py:147-260):

    triton.compile(ASTSource(fn, signature, constexprs), target=GPUTarget("cpu" | "npu" | "b200", 0, 0),
                   options={"pytorchsim_spec": <contract.kernel_spec JSON_FIELDS as JSON>})

runs Triton's own front end to TTIR, then this backend's "obj" stage lowers the kernel for the B200 executor:
the binary is the launch descriptor (desc.bin, the packed ptsim_desc of include/ptsim_b200.h) where the
reference yields a RISC-V ELF, and metadata["kernel_object"] holds the kernel.json text the launcher reads.

Behaviour the reference defines and this backend keeps:
  - without pytorchsim_spec the compile stops at TTIR: the binary is the TTIR text, the kernel object is empty,
    and a launch raises (driver._Launcher);
  - a program the lowering refuses is a RuntimeError naming the compiler gap, never OutOfResources (autotuning
    must not drop it as a capacity limit); any other failure of the stage is a RuntimeError too;
  - the backend's hash covers the pipeline's source, so a binary another pipeline built is never served from
    Triton's cache.
The B200 lowering reads the kernel's Python source (the @triton.jit function), not its TTIR: the obj stage
takes it from the ASTSource that triton.compile is compiling (Triton 3.6 calls each stage from compile(),
whose frame holds it as `src`), or from the spec's extra["source_path"] (a kernel file with a SPEC).
Options the reference uses for its simulator -- pytorchsim_tog (timing graph) and pytorchsim_target (machine
config) -- have no B200 meaning: a TOG request is refused, a target name is recorded and otherwise unused.

register() installs the backend into Triton (triton.backends.backends["pytorchsim"]) and makes it importable
under the reference's module names, triton.backends.pytorchsim.{compiler,driver}."""
import dataclasses
import functools
import hashlib
import json
import os
import shutil
import sys
import tempfile
from typing import Any, Dict, Tuple

from triton._C.libtriton import ir, passes
from triton.backends.compiler import BaseBackend, GPUTarget

HERE = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.dirname(HERE)
TARGETS = ("cpu", "npu", "b200")


@functools.lru_cache()
def _pipeline_fingerprint():
    """sha256 over the lowering's Python sources and the executor's kernel sources: Triton's cache key holds
    it, so a descriptor another pipeline built is never served."""
    digest = hashlib.sha256()
    roots = [os.path.join(PKG_ROOT, "pytorchsim_triton_compiler"), os.path.join(PKG_ROOT, "csrc")]
    for root in roots:
        for here, dirs, files in os.walk(root):
            dirs[:] = sorted(d for d in dirs if d not in ("__pycache__", "_lib"))
            for name in sorted(f for f in files if f.endswith((".py", ".cuh", ".cu", ".h"))):
                path = os.path.join(here, name)
                digest.update(os.path.relpath(path, PKG_ROOT).encode())
                with open(path, "rb") as f:
                    digest.update(f.read())
    return digest.hexdigest()


@dataclasses.dataclass(frozen=True)
class B200Options:
    debug: bool = False
    arch: Any = None
    num_warps: int = 0
    num_ctas: int = 0
    num_stages: int = 1
    enable_fp_fusion: bool = False
    cluster_dims: tuple = (1, 1, 1)
    shared: int = 0
    supported_fp8_dtypes: Tuple[str, ...] = ()
    deprecated_fp8_dot_operand_dtypes: Tuple[str, ...] = ()
    allow_fp8e4nv: bool = False
    allowed_dot_input_precisions: Tuple[str, ...] = ("ieee",)
    default_dot_input_precision: str = "ieee"
    max_num_imprecise_acc_default: int = 0
    sanitize_overflow: bool = True
    instrumentation_mode: str = ""
    backend_name: str = "pytorchsim"
    extern_libs: Any = None
    pytorchsim_spec: str = ""
    """JSON of contract.kernel_spec.JSON_FIELDS: what the lowering reads of the kernel beyond its source
    (argument roles and extents, grid, extra).  Empty: the backend stops at TTIR.  Part of the hash."""
    pytorchsim_keep_workdir: bool = False
    """Keep the stage's workdir (TTIR, kernel.json, desc.bin; also PYTORCHSIM_KEEP_WORKDIR=1); metadata["workdir"]
    names it."""
    pytorchsim_target: str = ""
    pytorchsim_tog: bool = False

    def hash(self):
        key = "_".join(f"{k}-{v}" for k, v in sorted(self.__dict__.items()))
        return hashlib.sha256(key.encode("utf-8")).hexdigest()


def _compiling_source():
    """The ASTSource triton.compile is compiling: the `src` local of the compile() frame that called this
    stage (None when the stage runs outside triton.compile)."""
    from triton.compiler.compiler import ASTSource
    f = sys._getframe(1)
    for _ in range(8):
        if f is None:
            return None
        src = f.f_locals.get("src")
        if isinstance(src, ASTSource):
            return src
        f = f.f_back
    return None


def lower_for_triton(ttir, spec_text, src=None, keep=False, metadata=None):
    """The descriptor of the kernel `src` (an ASTSource; or the spec's source file) under `spec_text`, with its
    kernel object, name and artifacts written into `metadata`."""
    from pytorchsim_triton_compiler.contract import kernel_object as ko
    from pytorchsim_triton_compiler.contract import kernel_spec as KS
    from pytorchsim_triton_compiler.contract.stop import Refused
    from pytorchsim_triton_compiler.targets.b200 import frontend as F
    from pytorchsim_triton_compiler.targets.b200 import lower as L
    metadata = {} if metadata is None else metadata
    work = tempfile.mkdtemp(prefix="pytorchsim-b200-")
    name = "kernel"
    try:
        ttir_path = os.path.join(work, "spec.ttir")
        with open(ttir_path, "w") as f:
            f.write(ttir)
        with open(os.path.join(work, "spec.json"), "w") as f:
            f.write(spec_text)
        spec = KS.spec_from_json(spec_text, ttir=ttir_path)
        name = spec.name
        fn = None
        if src is not None:
            fn = src.fn
            names = list(getattr(fn, "arg_names", []) or list(src.signature))
            spec.constexprs = {names[k[0]]: v for k, v in src.constants.items()
                               if isinstance(k, tuple) and len(k) == 1 and k[0] < len(names)
                               and isinstance(v, (int, float, bool))}
            if not spec.constexprs:
                spec.constexprs = {n: v for n, v in (getattr(src, "constexprs", None) or {}).items()}
        elif spec.extra.get("source_path"):
            own = KS.load_spec(spec.extra["source_path"])
            fn = F.load_kernel(own)
            spec.constexprs = dict(own.constexprs)
        else:
            raise RuntimeError(f"pytorchsim-triton-compiler (B200) lowers {name} from its Python source: compile it "
                               f"through triton.compile(ASTSource(...)) or name its kernel file in extra.source_path")
        try:
            lowered = L.lower(spec, fn=fn)
        except Refused as e:
            raise RuntimeError(f"pytorchsim-triton-compiler cannot lower {name} yet, a compiler gap "
                               f"({e.reason.value if hasattr(e.reason, 'value') else e.reason}), kept in {work}: {e}")
        ko.write(work, spec, lowered.summary, lowered.blob)
        with open(os.path.join(work, ko.MANIFEST)) as f:
            metadata["kernel_object"] = f.read()
        metadata["name"] = name
        metadata["artifacts"] = "{}"
        if keep:
            metadata["workdir"] = work
        return lowered.blob
    except RuntimeError:
        keep = True
        raise
    except Exception as e:  # noqa: BLE001 -- every other failure of the stage is the pipeline's
        keep = True
        raise RuntimeError(f"pytorchsim-triton-compiler failed on {name} (kept in {work}): {type(e).__name__}: {e}")
    finally:
        if not keep:
            shutil.rmtree(work, ignore_errors=True)


class CPUBackend(BaseBackend):
    """The backend (the reference's class name; the targets it accepts are the reference's "cpu" and "npu"
    and this build's "b200", all lowered for the B200 executor)."""
    binary_ext = "obj"

    @staticmethod
    def supports_target(target: GPUTarget):
        return target.backend in TARGETS

    def __init__(self, target: GPUTarget) -> None:
        super().__init__(target)

    def hash(self):
        return f"pytorchsim-b200-{_pipeline_fingerprint()}"

    def parse_options(self, opts) -> Any:
        args = {"arch": self.target.arch}
        args.update({k: opts[k] for k in B200Options.__dataclass_fields__ if k in opts})
        return B200Options(**args)

    def get_codegen_implementation(self, options):
        return {"min_dot_size": lambda lhs, rhs: (1, 1, 1)}

    def get_module_map(self) -> Dict[str, Any]:
        from triton.language.extra.cuda import libdevice
        return {"triton.language.extra.libdevice": libdevice}

    def load_dialects(self, ctx):
        return

    @staticmethod
    def make_ttir(mod, metadata, options):
        pm = ir.pass_manager(mod.context)
        pm.enable_debug()
        passes.common.add_inliner(pm)
        passes.ttir.add_rewrite_tensor_descriptor_to_pointer(pm)
        passes.common.add_canonicalizer(pm)
        passes.ttir.add_combine(pm)
        passes.ttir.add_reorder_broadcast(pm)
        passes.common.add_cse(pm)
        passes.common.add_symbol_dce(pm)
        passes.ttir.add_loop_unroll(pm)
        pm.run(mod, "make_ttir")
        return mod

    @staticmethod
    def make_obj(mod, metadata, options):
        if options.pytorchsim_tog:
            raise RuntimeError("pytorchsim_tog asks for the simulator's timing graph, which the B200 executor does not "
                               "build")
        keep = options.pytorchsim_keep_workdir or os.environ.get("PYTORCHSIM_KEEP_WORKDIR") == "1"
        return lower_for_triton(str(mod), options.pytorchsim_spec, _compiling_source(), keep, metadata)

    @staticmethod
    def make_ttir_only(mod, metadata):
        """A compile without pytorchsim_spec: the TTIR as the binary and no kernel object, so Triton accepts the
        kernel and a launch of it raises."""
        metadata["name"] = mod.get_entry_func_name()
        metadata["kernel_object"] = ""
        metadata["artifacts"] = "{}"
        return str(mod).encode()

    def pack_metadata(self, metadata):
        return ()

    def add_stages(self, stages, options, language=None):
        stages["ttir"] = lambda src, metadata: self.make_ttir(src, metadata, options)
        if options.pytorchsim_spec:
            stages["obj"] = lambda src, metadata: self.make_obj(src, metadata, options)
        else:
            stages["obj"] = lambda src, metadata: self.make_ttir_only(src, metadata)


def register():
    """Install the backend into this process's Triton (idempotent) and alias it as triton.backends.pytorchsim."""
    import types
    import triton.backends as TB
    from . import driver as D
    if "triton.backends.pytorchsim" not in sys.modules:
        pkg = types.ModuleType("triton.backends.pytorchsim")
        pkg.__path__ = []
        pkg.compiler = sys.modules[__name__]
        pkg.driver = D
        sys.modules["triton.backends.pytorchsim"] = pkg
        sys.modules["triton.backends.pytorchsim.compiler"] = sys.modules[__name__]
        sys.modules["triton.backends.pytorchsim.driver"] = D
    TB.backends["pytorchsim"] = TB.Backend(compiler=CPUBackend, driver=D.CPUDriver)
    return TB.backends["pytorchsim"]
