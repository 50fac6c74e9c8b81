"""Model-level API mirroring woolly-core: the Model trait (model/mod.rs:32-67),
InferenceSession::infer / infer_batch (session.rs:193-277) and
InferenceEngine (engine.rs:48-105), over the CUDA runtime in libwoolly_cuda.so.
"""
from __future__ import annotations

import ctypes as C
import os
from typing import Sequence

import numpy as np

from . import _lib
from ._lib import LOGITS_ALL, LOGITS_LAST, WoollyError, check, lib
from .gguf import config_dict


class Context:
    """One CUDA device with its own stream (wl_init)."""

    def __init__(self, device: int = 0):
        self._h = C.c_void_p()
        check(lib().wl_init(device, C.byref(self._h)))
        self.device = device

    def close(self):
        if self._h:
            lib().wl_ctx_free(self._h)
            self._h = None


def model_options(**kw) -> _lib.ModelOptions:
    o = _lib.ModelOptions()
    lib().wl_model_options_default(C.byref(o))
    for k, v in kw.items():
        if not hasattr(o, k):
            raise TypeError(f"unknown model option {k}")
        setattr(o, k, v)
    return o


def nccl_communicator(rank: int, world: int, group=None) -> int:
    """NCCL communicator for tensor parallelism across `world` ranks (one GPU
    each; call after torch.cuda.set_device).  Rank 0 draws the unique id
    (wl_nccl_unique_id) and the torch.distributed process group `group` (any
    backend; the default group when None) shares it.  Returns the handle to
    pass as CudaTransformer(..., tp_rank=rank, tp_size=world, nccl_comm=handle);
    release it with nccl_destroy() after the model is closed.
    """
    import torch.distributed as dist
    buf = (C.c_uint8 * 128)()
    if rank == 0:
        check(lib().wl_nccl_unique_id(buf))
    obj = [bytes(buf)]
    dist.broadcast_object_list(obj, src=0, group=group)
    uid = (C.c_uint8 * 128).from_buffer_copy(obj[0])
    comm = C.c_void_p()
    check(lib().wl_nccl_comm_init(world, uid, rank, C.byref(comm)))
    return comm.value


def nccl_destroy(comm: int) -> None:
    check(lib().wl_nccl_comm_destroy(C.c_void_p(comm)))


class CudaTransformer:
    """Drop-in for LazyTransformer behind woolly's Model trait.

    forward(input_ids) follows LazyTransformer::forward (lazy_transformer.rs:
    1155-1336): a full causal forward of the ids, returning seq_len * vocab
    logits (all positions, row-major).  Sessions keep a device KV cache for
    incremental decode.
    """

    def __init__(self, path: str, ctx: Context | None = None, **options):
        self.ctx = ctx or Context(options.pop("device", 0))
        self._own_ctx = ctx is None
        self._opts = model_options(**options)
        self._h = C.c_void_p()
        check(lib().wl_model_load_gguf(self.ctx._h, str(path).encode(), C.byref(self._opts),
                                       C.byref(self._h)))
        c = _lib.ModelConfig()
        check(lib().wl_model_get_config(self._h, C.byref(c)))
        self.config = config_dict(c)
        self._name = os.path.splitext(os.path.basename(path))[0]
        self._default: Session | None = None

    @classmethod
    def from_gguf(cls, path: str, **options) -> "CudaTransformer":
        return cls(path, **options)

    def close(self):
        if self._default is not None:
            self._default.close()
            self._default = None
        if self._h:
            lib().wl_model_free(self._h)
            self._h = None
        if self._own_ctx:
            self.ctx.close()

    # --- Model trait (model/mod.rs:32-67) ---
    def name(self) -> str:
        return self._name

    def model_type(self) -> str:
        return self.config["architecture"]

    @property
    def max_batch(self) -> int:
        """Most sessions one batched decode step takes (load option)."""
        return int(self._opts.max_batch)

    @property
    def max_context(self) -> int:
        """Tokens a session can hold (load option)."""
        return int(self._opts.max_context)

    def vocab_size(self) -> int:
        return self.config["vocab_size"]

    def context_length(self) -> int:
        return self.config["context_length"]

    def hidden_size(self) -> int:
        return self.config["hidden_size"]

    def num_layers(self) -> int:
        return self.config["num_layers"]

    def num_heads(self) -> int:
        return self.config["num_heads"]

    def forward(self, input_ids: Sequence[int]) -> np.ndarray:
        if len(input_ids) == 0:
            raise WoollyError(_lib.WL_ERR_INVALID_ARGUMENT, "Empty input tokens")
        if self._default is None:
            self._default = Session(self)
        self._default.reset()
        return self._default.infer(input_ids)

    def memory(self) -> tuple[int, int]:
        w, k = C.c_uint64(), C.c_uint64()
        check(lib().wl_model_memory(self._h, C.byref(w), C.byref(k)))
        return w.value, k.value

    def decode_kernel_count(self, n_sess: int) -> int:
        return lib().wl_decode_kernel_count(self._h, n_sess)

    # --- batched multi-session forward (wl_forward) ---
    def forward_sessions(self, sessions: Sequence["Session"], ids: Sequence[Sequence[int]],
                         all_logits: bool = False) -> list[np.ndarray]:
        n = len(sessions)
        counts = np.array([len(x) for x in ids], dtype=np.int32)
        flat = np.ascontiguousarray(np.concatenate([np.asarray(x, dtype=np.uint32) for x in ids]))
        V = self.vocab_size()
        rows = int(counts.sum()) if all_logits else n
        out = np.empty((rows, V), dtype=np.float32)
        arr = (C.c_void_p * n)(*[s._h for s in sessions])
        check(lib().wl_forward(self._h, arr, n, flat.ctypes.data, counts.ctypes.data,
                               out.ctypes.data, LOGITS_ALL if all_logits else LOGITS_LAST))
        if not all_logits:
            return [out[i] for i in range(n)]
        res, o = [], 0
        for c in counts:
            res.append(out[o:o + c])
            o += c
        return res

    def decode_step_device(self, sessions: Sequence["Session"], d_ids: int, d_logits: int,
                           stream: int = 0) -> None:
        """One batched decode step with device-resident ids/logits (raw pointers)."""
        arr = (C.c_void_p * len(sessions))(*[s._h for s in sessions])
        check(lib().wl_decode_step_device(self._h, arr, len(sessions), d_ids, d_logits, stream))


    def decode_sample(self, sessions: Sequence["Session"], ids: Sequence[int], temperature=0.0,
                      top_k=0, top_p=1.0, u=0.0) -> np.ndarray:
        """One batched decode step that returns the next token of every
        session, sampled on the GPU by the server's rules (wl_sample;
        inference.rs:441-483): the step's ids go to the device, only the
        sampled ids come back (4 bytes per session instead of a row of
        logits).  temperature / top_k / top_p / u are scalars or per-session
        sequences; u is the uniform draw of each session's sampling stream."""
        import torch
        from . import ops
        n = len(sessions)
        dev = torch.device("cuda", self.ctx.device)
        buf = getattr(self, "_ds_buf", None)
        if buf is None or buf[0].numel() < n:
            cap = max(n, self.max_batch)
            buf = (torch.empty(cap, dtype=torch.int32, pin_memory=True),
                   torch.empty(cap, dtype=torch.int32, device=dev),
                   torch.empty(cap, self.vocab_size(), dtype=torch.float32, device=dev),
                   torch.empty(cap, dtype=torch.int32, device=dev),
                   torch.empty(cap, dtype=torch.int32, pin_memory=True),
                   torch.empty(cap * 16, dtype=torch.uint8, device=dev))
            self._ds_buf = buf
        h_ids, d_ids, d_logits, d_next, h_next, d_prm = buf
        h_ids[:n] = torch.from_numpy(np.asarray(ids, dtype=np.int32))
        stream = torch.cuda.current_stream(dev)
        d_ids[:n].copy_(h_ids[:n], non_blocking=True)
        self.decode_step_device(sessions, d_ids.data_ptr(), d_logits.data_ptr(), stream.cuda_stream)
        ops.sample(d_logits[:n], temperature, top_k, top_p, u, out=d_next[:n], params=d_prm)
        h_next[:n].copy_(d_next[:n], non_blocking=True)
        stream.synchronize()
        return h_next[:n].numpy().copy()


class Session:
    """A device KV cache for one sequence (InferenceSession, session.rs:193-277)."""

    def __init__(self, model: CudaTransformer):
        self.model = model
        self._h = C.c_void_p()
        check(lib().wl_session_create(model._h, C.byref(self._h)))

    def close(self):
        if self._h:
            lib().wl_session_free(self._h)
            self._h = None

    def reset(self):
        check(lib().wl_session_reset(self._h))

    def __len__(self) -> int:
        return lib().wl_session_length(self._h)

    def infer(self, tokens: Sequence[int]) -> np.ndarray:
        """Appends tokens; returns their logits, flattened [len(tokens) * vocab]."""
        if len(tokens) == 0:
            raise WoollyError(_lib.WL_ERR_INVALID_ARGUMENT, "Empty input tokens")
        return self.model.forward_sessions([self], [tokens], all_logits=True)[0].reshape(-1)

    def infer_last(self, tokens: Sequence[int]) -> np.ndarray:
        return self.model.forward_sessions([self], [tokens], all_logits=False)[0]

    def infer_batch(self, batch: Sequence[Sequence[int]]) -> list[np.ndarray]:
        return [self.infer(t) for t in batch]


class InferenceSession:
    """InferenceSession (woolly-core/src/session.rs:118-330): one sequence's
    device KV cache plus the bookkeeping the reference keeps with it -- a
    string id, an active flag, the count of tokens processed and the token
    history.  Errors follow the reference: inference on a deactivated session
    (SESSION_INACTIVE) or with no tokens (empty input) raises WoollyError
    with WL_ERR_INVALID_ARGUMENT."""

    def __init__(self, model, session_id: str | None = None, backend=None):
        import uuid
        self.model = model
        self._id = session_id or str(uuid.uuid4())
        self._s = backend if backend is not None else Session(model)
        self._active = True
        self._history: list[int] = []

    def id(self) -> str:
        return self._id

    def is_active(self) -> bool:
        return self._active

    def tokens_processed(self) -> int:
        return len(self._history)

    def token_history(self) -> list[int]:
        return list(self._history)

    def infer(self, tokens: Sequence[int]) -> np.ndarray:
        """session.rs:193-258: appends the tokens to this session's context and
        returns their logits, flattened [len(tokens) * vocab]."""
        if not self._active:
            raise WoollyError(_lib.WL_ERR_INVALID_ARGUMENT, "Session is not active")
        if len(tokens) == 0:
            raise WoollyError(_lib.WL_ERR_INVALID_ARGUMENT, "Empty input tokens")
        out = self._s.infer(tokens)
        self._history += [int(t) for t in tokens]
        return out

    def infer_batch(self, batch: Sequence[Sequence[int]]) -> list[np.ndarray]:
        """session.rs:260-277: one infer() per item, in order."""
        return [self.infer(t) for t in batch]

    def clear(self) -> None:
        """session.rs:280-306: drops the history and the KV cache."""
        self._s.reset()
        self._history = []

    def deactivate(self) -> None:
        self._active = False

    def close(self) -> None:
        self._active = False
        self._s.close()


class SessionInfo(dict):
    """engine.rs SessionInfo: id, active, tokens_processed."""


class InferenceEngine:
    """InferenceEngine (woolly-core/src/engine.rs:15-246): holds one model and
    its sessions.  create_session() registers a new session; infer(tokens,
    session_id) runs on the named session (SESSION_NOT_FOUND if it is not
    registered) or, without an id, on a new registered session, as
    engine.rs:90-105 does; cleanup_sessions() drops inactive ones (closing
    their device caches)."""

    def __init__(self, session_factory=None):
        self.model = None
        self.sessions: list[InferenceSession] = []
        self._factory = session_factory

    def load_model(self, model) -> None:
        self.model = model

    def _need_model(self):
        if self.model is None:
            raise WoollyError(_lib.WL_ERR_INVALID_ARGUMENT, "No model loaded")
        return self.model

    def create_session(self, session_id: str | None = None) -> InferenceSession:
        m = self._need_model()
        backend = self._factory() if self._factory is not None else None
        s = InferenceSession(m, session_id, backend=backend)
        self.sessions.append(s)
        return s

    def find_session(self, session_id: str) -> InferenceSession:
        for s in self.sessions:
            if s.id() == session_id:
                return s
        raise WoollyError(_lib.WL_ERR_INVALID_ARGUMENT, f"Session not found: {session_id}")

    def infer(self, tokens: Sequence[int], session_id: str | None = None) -> np.ndarray:
        self._need_model()
        s = self.find_session(session_id) if session_id is not None else self.create_session()
        return s.infer(tokens)

    def list_sessions(self) -> list[SessionInfo]:
        return [SessionInfo(id=s.id(), active=s.is_active(), tokens_processed=s.tokens_processed())
                for s in self.sessions]

    def cleanup_sessions(self) -> None:
        keep = []
        for s in self.sessions:
            if s.is_active():
                keep.append(s)
            else:
                s.close()
        self.sessions = keep

    def model_info(self) -> dict | None:
        m = self.model
        if m is None:
            return None
        return dict(name=m.name(), model_type=m.model_type(), vocab_size=m.vocab_size(),
                    context_length=m.context_length(), hidden_size=m.hidden_size(),
                    num_layers=m.num_layers(), num_heads=m.num_heads())
