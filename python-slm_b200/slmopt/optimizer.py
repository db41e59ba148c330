"""Host-side mirror of the reference's optimizer interface over the C ABI.

``B200Adamw`` plays the role of ``CanonicalAdamw`` / ``FullModelState``
(src/train/trainer.rs:193-321, src/train/full_state.rs:196-520) with the state
resident in HBM; ``B200TrainerBackend`` is the ``TrainerBackend`` surface the
trainer calls (src/train/trainer.rs:510-522): ``apply_update``, ``snapshot``
and ``restore``.  Every numeric operation runs in libslmopt.so.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib
from .layout import GqaDimensions, TensorTable

# Artifact roles and paths of the five-artifact codec (src/train/full_state.rs:27-36).
ARTIFACTS = (
    ("parameters_bf16", "model/parameters.bf16", _lib.ROLE_PARAMETERS_BF16, np.uint16),
    ("master_parameters_fp32", "optimizer/master.f32", _lib.ROLE_MASTER_F32, np.float32),
    ("adamw_first_moments_fp32", "optimizer/adamw-m1.f32", _lib.ROLE_MOMENT1_F32, np.float32),
    ("adamw_second_moments_fp32", "optimizer/adamw-m2.f32", _lib.ROLE_MOMENT2_F32, np.float32),
)


@dataclass
class StepOptions:
    """Python view of slm_step_config; defaults are OPT-001 (oracle.rs:469-484)."""

    learning_rate: float = 3e-4
    one_based_update: int = 1
    beta1: float = 0.9
    beta2: float = 0.95
    epsilon: float = 1e-8
    decay_weight: float = 0.1
    no_decay_weight: float = 0.0
    max_grad_norm: float = 1.0
    apply_clip: bool = True
    min_clip_accept: float = 0.0
    nonfinite_policy: int = _lib.NONFINITE_SKIP
    loss_scale_mode: int = _lib.SCALE_STATIC
    static_loss_scale: float = 1.0
    growth_interval: int = 2000

    def to_c(self) -> _lib.StepConfig:
        c = _lib.StepConfig()
        c.learning_rate = self.learning_rate
        c.one_based_update = self.one_based_update
        c.beta1 = self.beta1
        c.beta2 = self.beta2
        c.epsilon = self.epsilon
        c.decay_weight = self.decay_weight
        c.no_decay_weight = self.no_decay_weight
        c.max_grad_norm = self.max_grad_norm
        c.apply_clip = 1 if self.apply_clip else 0
        c.min_clip_accept = self.min_clip_accept
        c.nonfinite_policy = self.nonfinite_policy
        c.loss_scale_mode = self.loss_scale_mode
        c.static_loss_scale = self.static_loss_scale
        c.growth_interval = self.growth_interval
        return c


def _grad_pointer(grads):
    """(pointer, dtype code, memory kind, element count, keep-alive) for a
    torch tensor (device or host) or a numpy array (host)."""
    if isinstance(grads, np.ndarray):
        if grads.dtype == np.float32:
            dt = _lib.DTYPE_F32
        elif grads.dtype == np.uint16:
            dt = _lib.DTYPE_BF16
        else:
            raise TypeError("host gradients must be float32 or uint16 (bf16 bits)")
        arr = np.ascontiguousarray(grads)
        return arr.ctypes.data, dt, _lib.MEMORY_HOST, arr.size, arr
    import torch  # plumbing only: device memory and streams

    if not isinstance(grads, torch.Tensor):
        raise TypeError("gradients must be a numpy array or a torch tensor")
    if not grads.is_contiguous():
        raise ValueError("gradients must be contiguous")
    if grads.dtype == torch.float32:
        dt = _lib.DTYPE_F32
    elif grads.dtype in (torch.bfloat16, torch.int16, torch.uint16):
        dt = _lib.DTYPE_BF16
    else:
        raise TypeError("gradients must be float32 or bfloat16")
    mem = _lib.MEMORY_DEVICE if grads.is_cuda else _lib.MEMORY_HOST
    return grads.data_ptr(), dt, mem, grads.numel(), grads


class B200Adamw:
    """Device-resident AdamW state for one PARAM-001 tensor table."""

    def __init__(self, table: TensorTable, device: int = 0):
        self.lib = _lib.load()
        self.table = table
        self.device = device
        specs = (_lib.TensorSpec * len(table))()
        self._names = [n.encode() for n in table.names]
        for i, (name, n, dec) in enumerate(zip(self._names, table.elements, table.decay)):
            specs[i].name = name
            specs[i].elements = n
            specs[i].weight_decay = 1 if dec else 0
        h = ctypes.c_void_p()
        _lib.check(self.lib.slm_opt_create(specs, len(table), device, ctypes.byref(h)))
        self._h = h
        self.P = int(self.lib.slm_opt_parameter_count(h))

    @classmethod
    def from_dimensions(cls, dims: GqaDimensions, device: int = 0) -> "B200Adamw":
        return cls(TensorTable.from_dimensions(dims), device)

    # ---- lifetime -------------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "_h", None):
            self.lib.slm_opt_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _check(self, status: int) -> None:
        _lib.check(status, self._h)

    # ---- state ------------------------------------------------------------------
    def init_master(self, master: np.ndarray) -> None:
        m = np.ascontiguousarray(master, dtype=np.float32)
        if m.size != self.P:
            raise ValueError("master must have one value per parameter")
        self._check(self.lib.slm_opt_init_master(self._h, m.ctypes.data, None))

    def load_state(self, master: np.ndarray, moment: np.ndarray, variance: np.ndarray,
                   bf16: np.ndarray, validate: bool = True) -> None:
        for role, arr, dt in ((_lib.ROLE_MASTER_F32, master, np.float32),
                              (_lib.ROLE_MOMENT1_F32, moment, np.float32),
                              (_lib.ROLE_MOMENT2_F32, variance, np.float32),
                              (_lib.ROLE_PARAMETERS_BF16, bf16, np.uint16)):
            a = np.ascontiguousarray(arr, dtype=dt)
            self._check(self.lib.slm_opt_restore(self._h, role, a.ctypes.data, a.nbytes))
        if validate:
            self._check(self.lib.slm_opt_validate_state(self._h))

    def read_state(self) -> dict[str, np.ndarray]:
        out = {}
        for key, role, dt in (("master", _lib.ROLE_MASTER_F32, np.float32),
                              ("moment", _lib.ROLE_MOMENT1_F32, np.float32),
                              ("variance", _lib.ROLE_MOMENT2_F32, np.float32),
                              ("bf16", _lib.ROLE_PARAMETERS_BF16, np.uint16)):
            a = np.empty(self.P, dtype=dt)
            self._check(self.lib.slm_opt_snapshot(self._h, role, a.ctypes.data, a.nbytes))
            out[key] = a
        return out

    def device_buffer(self, role: int) -> int:
        p = ctypes.c_void_p()
        self._check(self.lib.slm_opt_device_buffer(self._h, role, ctypes.byref(p)))
        return int(p.value)

    def validate(self) -> None:
        self._check(self.lib.slm_opt_validate_state(self._h))

    def export_weights_f32(self, out=None, stream=None):
        """The bf16 weights as an f32 CUDA tensor of P elements (the values the
        reference's graph reload uploads), written on the device on `stream`."""
        import torch

        P = self.P
        if out is None:
            out = torch.empty(P, dtype=torch.float32, device=f"cuda:{self.device}")
        if out.dtype != torch.float32 or not out.is_cuda or not out.is_contiguous() or \
                out.numel() != P:
            raise ValueError("out must be a contiguous f32 CUDA tensor of P elements")
        self._check(self.lib.slm_opt_export_weights_f32(self._h, out.data_ptr(), P,
                                                        _stream_handle(stream)))
        return out

    def state_sha256(self) -> str:
        buf = ctypes.create_string_buffer(65)
        self._check(self.lib.slm_opt_state_sha256(self._h, buf))
        return buf.value.decode()

    # ---- loss scaler ----------------------------------------------------------------
    def set_loss_scale(self, scale: float, good_steps: int = 0) -> None:
        self._check(self.lib.slm_opt_set_loss_scale(self._h, scale, good_steps))

    def loss_scale(self) -> tuple[float, int]:
        s, g = ctypes.c_float(), ctypes.c_uint32()
        self._check(self.lib.slm_opt_get_loss_scale(self._h, ctypes.byref(s), ctypes.byref(g)))
        return s.value, g.value

    # ---- the step ----------------------------------------------------------------------
    def step(self, grads, options: StepOptions | None = None, stream=None,
             wait: bool = True) -> _lib.StepResult | None:
        """Fused step over P gradients (torch device tensor or host array).

        With ``wait`` the call blocks and returns the StepResult (raising
        SlmError on a failed status); otherwise it only enqueues on ``stream``.
        """
        ptr, dt, mem, n, keep = _grad_pointer(grads)
        if n != self.P:
            raise ValueError(f"expected {self.P} gradients, got {n}")
        cfg = (options or StepOptions()).to_c()
        s = _stream_handle(stream)
        if wait:
            res = _lib.StepResult()
            st = self.lib.slm_opt_step(self._h, ptr, dt, mem, ctypes.byref(cfg), ctypes.byref(res), s)
            del keep
            self._check(st)
            return res
        self._check(self.lib.slm_opt_step(self._h, ptr, dt, mem, ctypes.byref(cfg), None, s))
        return None

    def upload(self, grads) -> int:
        """Start copying host gradients (numpy array or CPU tensor, pinned for
        an asynchronous copy) into a device slot on the handle's copy stream;
        returns the slot for step_uploaded.  The buffer is kept alive here
        until the slot is reused (which first waits for the step that read
        it), or the handle is closed."""
        ptr, dt, mem, n, keep = _grad_pointer(grads)
        if mem != _lib.MEMORY_HOST:
            raise ValueError("upload takes host gradients")
        if n != self.P:
            raise ValueError(f"expected {self.P} gradients, got {n}")
        slot = ctypes.c_int()
        self._check(self.lib.slm_opt_upload_gradients(self._h, ptr, dt, ctypes.byref(slot)))
        if not hasattr(self, "_upload_keep"):
            self._upload_keep = [None, None]
        self._upload_keep[slot.value] = keep
        return slot.value

    def step_uploaded(self, slot: int, options: StepOptions | None = None, stream=None,
                      wait: bool = True) -> _lib.StepResult | None:
        """The fused step over the gradients of an upload slot (see step)."""
        cfg = (options or StepOptions()).to_c()
        s = _stream_handle(stream)
        if wait:
            res = _lib.StepResult()
            self._check(self.lib.slm_opt_step_uploaded(self._h, slot, ctypes.byref(cfg),
                                                       ctypes.byref(res), s))
            return res
        self._check(self.lib.slm_opt_step_uploaded(self._h, slot, ctypes.byref(cfg), None, s))
        return None

    def norm_pass(self, grads, options: StepOptions | None = None, stream=None):
        """Enqueue the unscale / non-finite / norm / clip pass; returns the
        keep-alive object that must outlive the matching update_pass."""
        ptr, dt, mem, n, keep = _grad_pointer(grads)
        if n != self.P:
            raise ValueError(f"expected {self.P} gradients, got {n}")
        cfg = (options or StepOptions()).to_c()
        self._check(self.lib.slm_opt_norm_pass(self._h, ptr, dt, mem, ctypes.byref(cfg),
                                               _stream_handle(stream)))
        return keep

    def accumulate(self, acc, micro, overwrite: bool = False, stream=None) -> None:
        """acc (device f32[P]) += micro (device f32 or bf16 [P]), or acc = micro."""
        ptr, dt, mem, n, keep = _grad_pointer(micro)
        if mem != _lib.MEMORY_DEVICE or not acc.is_cuda:
            raise ValueError("accumulate works on device tensors")
        if n != self.P or acc.numel() != self.P:
            raise ValueError(f"expected {self.P} elements")
        _lib.check(self.lib.slm_grad_accumulate(acc.data_ptr(), ptr, dt, n, 1 if overwrite else 0,
                                                _stream_handle(stream)))

    def norm_pass_accumulate(self, acc, micro, options: StepOptions | None = None,
                             overwrite: bool = False, stream=None):
        """Last micro-batch: acc += micro fused with the norm pass over acc;
        follow with update_pass().  Returns the keep-alive for micro."""
        ptr, dt, mem, n, keep = _grad_pointer(micro)
        if n != self.P or acc.numel() != self.P:
            raise ValueError(f"expected {self.P} elements")
        cfg = (options or StepOptions()).to_c()
        self._check(self.lib.slm_opt_norm_pass_accumulate(
            self._h, acc.data_ptr(), ptr, dt, mem, 1 if overwrite else 0, ctypes.byref(cfg),
            _stream_handle(stream)))
        return keep

    def update_pass(self, options: StepOptions | None = None, stream=None) -> None:
        cfg = (options or StepOptions()).to_c()
        self._check(self.lib.slm_opt_update_pass(self._h, ctypes.byref(cfg),
                                                 _stream_handle(stream)))

    def read_result(self) -> _lib.StepResult:
        res = _lib.StepResult()
        self._check(self.lib.slm_opt_read_result(self._h, ctypes.byref(res)))
        return res

    def phase_timing(self, enable: bool = True) -> None:
        """Record per-phase device times of each step (clears earlier sums).
        Each step then waits for the previous one: keep it off in timed runs."""
        self._check(self.lib.slm_opt_phase_timing(self._h, 1 if enable else 0))

    def phase_times(self) -> tuple[dict[str, float], int]:
        """Mean ms per phase of the steps timed since phase_timing(True), and
        how many steps that was."""
        out = (ctypes.c_double * 8)()
        n, steps = ctypes.c_uint32(), ctypes.c_uint64()
        self._check(self.lib.slm_opt_phase_times(self._h, out, 8, ctypes.byref(n),
                                                 ctypes.byref(steps)))
        names = [self.lib.slm_opt_phase_name(self._h, i).decode() for i in range(n.value)]
        return {name: out[i] for i, name in enumerate(names)}, int(steps.value)

    def apply_normalized_clipped_gradients(self, gradients: np.ndarray, learning_rate: float,
                                           one_based_update: int, valid_targets: int = 0,
                                           with_sha: bool = True) -> str | None:
        """CanonicalAdamw::apply_normalized_clipped_gradients (trainer.rs:222-295)."""
        g = np.ascontiguousarray(gradients, dtype=np.float32)
        buf = ctypes.create_string_buffer(65) if with_sha else None
        self._check(self.lib.slm_opt_apply_update(self._h, g.ctypes.data, g.size,
                                                  ctypes.c_float(learning_rate),
                                                  one_based_update, valid_targets, buf))
        return buf.value.decode() if with_sha else None


def gradient_clip_scale(gradients, stream=None, parallel: bool = True) -> tuple[int, float, float]:
    """The reference's gradient_clip_scale (src/model/oracle.rs:486-507) of a
    contiguous f32 CUDA tensor, bit for bit, on the device:
    (status, sequential f32 sum of squares, clip scale).  parallel=True
    summarises the windows on every SM (slm_gradient_clip_scale_ws, with a
    workspace allocated here); False streams them through one CTA
    (slm_gradient_clip_scale).  Waits for the result."""
    import torch

    if not (gradients.is_cuda and gradients.dtype == torch.float32 and gradients.is_contiguous()):
        raise ValueError("gradients must be a contiguous f32 CUDA tensor")
    lib = _lib.load()
    n = gradients.numel()
    out = torch.zeros(ctypes.sizeof(_lib.ClipResult), dtype=torch.uint8, device=gradients.device)
    if parallel:
        ws_bytes = int(lib.slm_gradient_clip_workspace_bytes(n))
        ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=gradients.device)
        _lib.check(lib.slm_gradient_clip_scale_ws(gradients.data_ptr(), n, ws.data_ptr(),
                                                  ws_bytes, out.data_ptr(),
                                                  _stream_handle(stream)))
    else:
        _lib.check(lib.slm_gradient_clip_scale(gradients.data_ptr(), n, out.data_ptr(),
                                               _stream_handle(stream)))
    res = _lib.ClipResult.from_buffer_copy(out.cpu().numpy().tobytes())
    if res.kernel_error:
        raise _lib.SlmError(_lib.SLM_ERR_INTERNAL, "the clip scale kernel's copy pipeline stalled")
    return int(res.status), float(res.sum_squares), float(res.clip_scale)


def _stream_handle(stream) -> int | None:
    if stream is None:
        return None
    if isinstance(stream, int):
        return stream
    return int(stream.cuda_stream)  # torch.cuda.Stream


class B200TrainerBackend:
    """``TrainerBackend`` optimizer surface (src/train/trainer.rs:510-522) as
    ``CudaTrainerBackend`` implements it (src/train/cuda_backend.rs:240-308),
    with the state kept on the device instead of re-uploaded after each update."""

    def __init__(self, dims: GqaDimensions, device: int = 0):
        self.dims = dims
        self.optimizer = B200Adamw.from_dimensions(dims, device)

    def apply_update(self, normalized_clipped_gradients: np.ndarray, learning_rate: float,
                     one_based_update: int, valid_targets: int) -> str:
        return self.optimizer.apply_normalized_clipped_gradients(
            normalized_clipped_gradients, learning_rate, one_based_update, valid_targets)

    def snapshot(self) -> list[tuple[str, str, bytes]]:
        """The four optimizer artifacts as (role, relative_path, bytes)."""
        st = self.optimizer.read_state()
        keys = {"parameters_bf16": "bf16", "master_parameters_fp32": "master",
                "adamw_first_moments_fp32": "moment", "adamw_second_moments_fp32": "variance"}
        return [(role, path, st[keys[role]].tobytes()) for role, path, _, _ in ARTIFACTS]

    def restore(self, artifacts) -> None:
        by_role = {role: (path, data) for role, path, data in artifacts}
        arrays = {}
        for role, path, _, dt in ARTIFACTS:
            if role not in by_role:
                raise _lib.SlmError(_lib.SLM_ERR_E1_STATE_ARTIFACT_INVALID,
                                    f"the checkpoint omits the {role} artifact")
            got_path, data = by_role[role]
            if got_path != path:
                raise _lib.SlmError(_lib.SLM_ERR_E1_STATE_ARTIFACT_INVALID,
                                    f"the {role} artifact is not at its closed relative path")
            arrays[role] = np.frombuffer(data, dtype=dt)
        self.optimizer.load_state(arrays["master_parameters_fp32"],
                                  arrays["adamw_first_moments_fp32"],
                                  arrays["adamw_second_moments_fp32"],
                                  arrays["parameters_bf16"])

    def state_sha256(self) -> str:
        return self.optimizer.state_sha256()
