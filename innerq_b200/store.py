"""GPU-resident store of one side (K or V) of one InnerQ cache layer.

Token order matches the reference layer (``src/innerq/cache.py:235-276``):
``[sink (dtype) | quantized middle (packed) | recent window (dtype)]``.

* sink:   ``[B, H, n_sink, D]`` fixed at prefill (``cache.py:135-155``).
* middle: packed 2/3/4-bit tiles of 32 tokens plus per-group scales / zero
          points, written in place by ``innerq_quant_pack`` at the append
          position (the reference ``torch.cat``\\ s onto the store,
          ``cache.py:337-339, 363-365``).  Capacity grows by doubling.
* recent: a FIFO window ``[B, H, cap, D]`` in the dtype; the oldest
          ``flush_size`` tokens are quantized and popped when the window holds
          at least ``flush_size`` (``cache.py:283-307``).

All compute goes through ``libinnerq_b200.so``; torch only allocates and
copies device memory.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib

D_SUPPORTED = 128


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float16:
        return _lib.DT_F16
    if dt == torch.bfloat16:
        return _lib.DT_BF16
    raise TypeError(f"innerq_b200 kernels take float16 or bfloat16 tensors, got {dt}")


try:
    _raw_stream = torch._C._cuda_getCurrentRawStream
except AttributeError:  # pragma: no cover - older torch
    _raw_stream = None


def stream_ptr(device: torch.device) -> int:
    """cudaStream_t of the current torch stream on `device` (as an int)."""
    if _raw_stream is not None:
        return _raw_stream(device.index if device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(t: torch.Tensor, what: str):
    if not t.is_cuda:
        raise RuntimeError(f"{what} must be a CUDA tensor: innerq_b200 has no CPU path")


def _ptr(t):
    return None if t is None else t.data_ptr()


class PackedSide:
    """One of K / V of one layer."""

    def __init__(self, role: int, bits: int, group: int, mode: int, over_token: bool,
                 w_sink: int, w_recent: int, flush: int, normalize: bool = False):
        self.role, self.bits, self.group, self.mode = role, bits, group, mode
        self.over_token = bool(over_token)
        self.w_sink, self.w_recent, self.flush = w_sink, w_recent, flush
        self.normalize = normalize
        self.quantize = bits < 16
        self.dtype = self.device = None
        self.B = self.H = self.D = 0
        self.sink = None
        self.codes = self.scale = self.zero = None
        self.cap_tiles = 0
        self.n_q = 0
        self.norm_f = None            # [B, H, D] dtype
        self._rbuf = None             # recent FIFO buffer [B, H, cap, D]
        self._r0 = 0
        self._rn = 0
        self.headroom = 1024          # tokens of spare packed capacity per growth
        self._g0 = None               # graph mode: (n_q, n_recent, r0) at step 0

    # ------------------------------------------------------------- geometry
    def _check_supported(self):
        if not self.quantize:
            return
        if self.bits not in (1, 2, 3, 4) or (self.bits == 1 and self.mode == _lib.SYM):
            raise NotImplementedError(f"{self.bits}-bit codes are not built (2, 3, 4; 1 asymmetric)")
        if self.group not in (32, 64, 128):
            raise NotImplementedError(f"group size {self.group} is not built (32, 64, 128 are)")
        if self.D != D_SUPPORTED:
            raise NotImplementedError(f"head_dim {self.D} is not built (128 is)")

    @property
    def fusable(self) -> bool:
        """The fused decode attention reads this side's layout: keys grouped
        over channels, or over tokens (KIVI) without key normalisation; values
        over tokens (the InnerQ default) or over channels (group sizes checked
        by the layer)."""
        if not self.quantize:
            return True
        return self.role == _lib.ROLE_V or not self.over_token or not self.normalize

    @property
    def n_sink(self) -> int:
        return 0 if self.sink is None else self.sink.shape[2]

    @property
    def n_recent(self) -> int:
        return self._rn

    @property
    def recent(self) -> torch.Tensor:
        return self._rbuf[:, :, self._r0:self._r0 + self._rn]

    @property
    def n_tokens(self) -> int:
        return self.n_sink + self.n_q + self.n_recent

    # ------------------------------------------------------------ storage
    def _alloc_store(self, tokens: int):
        tb = _lib.load().innerq_tile_bytes(self.bits)
        cap_tiles = max(4, (tokens + 31) // 32)
        if self.over_token:
            cap_tiles = (cap_tiles * 32 + self.group - 1) // self.group * self.group // 32
        B, H, D = self.B, self.H, self.D
        # values grouped over channels OR their codes into shared words: zero-fill
        alloc = torch.zeros if (self.role == _lib.ROLE_V and not self.over_token) else torch.empty
        codes = alloc((B, H, cap_tiles, tb), dtype=torch.uint8, device=self.device)
        if self.over_token:
            sshape = (B, H, cap_tiles * 32 // self.group, D)
        else:
            sshape = (B, H, cap_tiles * 32, D // self.group)
        scale = torch.empty(sshape, dtype=self.dtype, device=self.device)
        zero = torch.empty(sshape, dtype=self.dtype, device=self.device) if self.mode == _lib.ASYM else None
        if self.codes is not None and self.n_q > 0:
            nt = (self.n_q + 31) // 32
            codes[:, :, :nt].copy_(self.codes[:, :, :nt])
            ns = (self.n_q // self.group) if self.over_token else nt * 32
            scale[:, :, :ns].copy_(self.scale[:, :, :ns])
            if zero is not None:
                zero[:, :, :ns].copy_(self.zero[:, :, :ns])
        self.codes, self.scale, self.zero, self.cap_tiles = codes, scale, zero, cap_tiles

    def reserve(self, n_quantized: int):
        """Make room for n_quantized packed tokens (grows by doubling)."""
        if self.codes is None:
            self._alloc_store(n_quantized + self.headroom)
        elif n_quantized > self.cap_tiles * 32:
            cap = self.cap_tiles * 32
            self._alloc_store(max(n_quantized, cap + max(self.headroom, cap // 4)))

    def _recent_reserve(self, n_new: int):
        need = self._rn + n_new
        if self._rbuf is not None and self._r0 + need <= self._rbuf.shape[2]:
            return
        # slack so the FIFO compacts rarely (once per ~1000 appended tokens)
        cap = max(need, self.w_recent + self.flush + 1024, 2 * self._rn)
        if self._rbuf is None or cap > self._rbuf.shape[2]:
            buf = torch.empty((self.B, self.H, cap, self.D), dtype=self.dtype, device=self.device)
        else:
            buf = torch.empty_like(self._rbuf)
        if self._rn:
            buf[:, :, :self._rn].copy_(self.recent)
        self._rbuf, self._r0 = buf, 0

    def _push_recent(self, x: torch.Tensor):
        self._recent_reserve(x.shape[2])
        self._rbuf[:, :, self._r0 + self._rn:self._r0 + self._rn + x.shape[2]].copy_(x)
        self._rn += x.shape[2]

    # ---------------------------------------------------------- quantize
    def _quantize(self, x: torch.Tensor):
        """Quantize-and-pack x [B, H, T, D] at the append position."""
        T = x.shape[2]
        if T == 0:
            return
        if self.over_token:
            assert T % self.group == 0  # quant.py:99
        if self.normalize and self.norm_f is None:
            # cache.py:124: factor from the first chunk that gets quantized
            self.norm_f = torch.empty((self.B, self.H, self.D), dtype=self.dtype, device=self.device)
            _lib.call("innerq_norm_factor", x.data_ptr(), dtype_code(self.dtype), self.B, self.H, T,
                      self.D, x.stride(0), x.stride(1), x.stride(2), self.norm_f.data_ptr(),
                      stream_ptr(self.device))
        self.reserve(self.n_q + T)
        if x.stride(3) != 1 or (not self.over_token and (x.data_ptr() % 8 or x.stride(0) % 4 or x.stride(1) % 4
                                                        or x.stride(2) % 4)):
            x = x.contiguous()
        _lib.call("innerq_quant_pack", x.data_ptr(), dtype_code(self.dtype), self.B, self.H, T, self.D,
                  x.stride(0), x.stride(1), x.stride(2), self.bits, self.group, self.mode, self.role,
                  int(self.over_token), _ptr(self.norm_f if self.normalize else None),
                  self.codes.data_ptr(), self.scale.data_ptr(), _ptr(self.zero), self.cap_tiles,
                  self.n_q, stream_ptr(self.device))
        self.n_q += T

    # ---------------------------------------------------- reference logic
    def prefill(self, x: torch.Tensor):
        """Lazy initialisation (cache.py:135-185, 187-210) from prefill tokens."""
        require_cuda(x, "key/value states")
        self.dtype, self.device = x.dtype, x.device
        dtype_code(self.dtype)
        self.B, self.H, T, self.D = x.shape
        self._check_supported()
        n_sink = min(self.w_sink, T) if self.quantize else 0
        # a copy, never a view: even an empty slice would keep the whole
        # prefill tensor alive for the life of the cache
        self.sink = x[:, :, :n_sink].clone(memory_format=torch.contiguous_format)
        x = x[:, :, n_sink:]
        T = x.shape[2]
        if self.quantize:
            r = min(self.w_recent, T)
            if self.over_token:
                while (T - r) % self.flush != 0:
                    r -= 1
        else:
            r = T
        nq = T - r
        self._push_recent(x[:, :, nq:])
        if self.quantize and nq > 0:
            self._quantize(x[:, :, :nq])

    def append(self, x: torch.Tensor):
        """One decode update (cache.py:283-307 then 314-380)."""
        require_cuda(x, "key/value states")
        self._push_recent(x)
        if self.quantize and self._rn >= self.flush:
            out = self._rbuf[:, :, self._r0:self._r0 + self.flush]
            self._quantize(out)
            self._r0 += self.flush
            self._rn -= self.flush

    # ------------------------------------------------------------- views
    def materialize(self) -> torch.Tensor:
        """[sink | dequant(middle) | recent] in the dtype (cache.py:235-281)."""
        out = torch.empty((self.B, self.H, self.n_tokens, self.D), dtype=self.dtype, device=self.device)
        ns, nq = self.n_sink, self.n_q
        if ns:
            out[:, :, :ns].copy_(self.sink)
        if nq:
            mid = out[:, :, ns:ns + nq]
            _lib.call("innerq_dequant", self.codes.data_ptr(), self.scale.data_ptr(), _ptr(self.zero),
                      dtype_code(self.dtype), self.B, self.H, 0, nq, self.D, self.bits, self.group,
                      self.mode, self.role, int(self.over_token), self.cap_tiles,
                      _ptr(self.norm_f if self.normalize else None), mid.data_ptr(),
                      mid.stride(0), mid.stride(1), mid.stride(2), stream_ptr(self.device))
        if self._rn:
            out[:, :, ns + nq:].copy_(self.recent)
        return out

    def ref_views(self):
        """(int32 codes, scale, sign | zero) exactly as quant.py returns them for
        the quantized tokens, or (None, None, None)."""
        if self.n_q == 0:
            return None, None, None
        B, H, D, n = self.B, self.H, self.D, self.n_q
        codes = torch.empty((B, H, n, D), dtype=torch.int32, device=self.device)
        if self.over_token:
            sshape = (B, H, n // self.group, D)
        else:
            sshape = (B, H, n, D // self.group)
        scale = torch.empty(sshape, dtype=self.dtype, device=self.device)
        if self.mode == _lib.ASYM:
            zs = torch.empty(sshape, dtype=self.dtype, device=self.device)
            sign = None
        else:
            zs = torch.empty((B, H, n, D), dtype=self.dtype, device=self.device)
            sign = zs
        _lib.call("innerq_unpack_ref", self.codes.data_ptr(), self.scale.data_ptr(), _ptr(self.zero),
                  dtype_code(self.dtype), B, H, 0, n, D, self.bits, self.group, self.mode, self.role,
                  int(self.over_token), self.cap_tiles, codes.data_ptr(), _ptr(sign),
                  scale.data_ptr(), _ptr(zs if sign is None else None), stream_ptr(self.device))
        return codes, scale, zs

    # ------------------------------------------------------- serialisation
    _CONFIG_KEYS = ("role", "bits", "group", "mode", "over_token", "w_sink", "w_recent", "flush",
                    "normalize")

    def state_dict(self) -> dict:
        """This side's content as host tensors and plain values: the config it
        was built with, the sink, the packed tiles and scales / zero points
        actually in use (not the spare capacity), the normalisation factor and
        the recent window.  The tiles keep their on-device layout (the packed
        format of ``csrc/common.cuh``), so a restored side continues bit for
        bit where this one stopped."""
        if self._g0 is not None:
            raise RuntimeError("cannot serialise a store in graph mode (call graph_end first)")
        d = {k: getattr(self, k) for k in self._CONFIG_KEYS}
        d["initialized"] = self.dtype is not None
        if not d["initialized"]:
            return d
        d["dtype"] = str(self.dtype).replace("torch.", "")
        d["shape"] = (self.B, self.H, self.D)
        d["n_q"] = self.n_q
        d["sink"] = None if self.sink is None else self.sink.cpu()
        d["recent"] = self.recent.cpu() if self._rbuf is not None else None
        d["norm_f"] = None if self.norm_f is None else self.norm_f.cpu()
        d["codes"] = d["scale"] = d["zero"] = None
        if self.quantize and self.n_q:
            nt = (self.n_q + 31) // 32
            ns = (self.n_q // self.group) if self.over_token else nt * 32
            d["codes"] = self.codes[:, :, :nt].cpu()
            d["scale"] = self.scale[:, :, :ns].cpu()
            d["zero"] = None if self.zero is None else self.zero[:, :, :ns].cpu()
        return d

    def load_state_dict(self, d: dict, device) -> None:
        """Restore a side written by state_dict() onto `device` (a CUDA
        device; None: the current one).  The config must match the one this
        side was built with."""
        for k in self._CONFIG_KEYS:
            if d.get(k) != getattr(self, k):
                raise ValueError(f"saved cache store has {k}={d.get(k)!r}, this layer {getattr(self, k)!r}")
        self.codes = self.scale = self.zero = None
        self.cap_tiles = self.n_q = 0
        self._rbuf, self._r0, self._rn = None, 0, 0
        self.norm_f = None
        if not d["initialized"]:
            self.dtype = self.device = self.sink = None
            return
        device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        if device.type != "cuda":
            raise RuntimeError("innerq_b200 stores live on a CUDA device: it has no CPU path")
        self.dtype = getattr(torch, d["dtype"])
        dtype_code(self.dtype)
        self.device = device
        self.B, self.H, self.D = d["shape"]
        self._check_supported()
        self.sink = None if d["sink"] is None else d["sink"].to(device=device, dtype=self.dtype).contiguous()
        if d["norm_f"] is not None:
            self.norm_f = d["norm_f"].to(device).contiguous()
        n_q = int(d["n_q"])
        if self.quantize and n_q:
            self._alloc_store(n_q + self.headroom)
            nt, ns = d["codes"].shape[2], d["scale"].shape[2]
            self.codes[:, :, :nt].copy_(d["codes"])
            self.scale[:, :, :ns].copy_(d["scale"])
            if self.zero is not None:
                self.zero[:, :, :ns].copy_(d["zero"])
        self.n_q = n_q
        if d["recent"] is not None:
            self._push_recent(d["recent"].to(device))

    # ---------------------------------------------------------- graph mode
    def graph_begin(self, max_steps: int):
        """Prepare for up to `max_steps` decode steps replayed from a CUDA
        graph: the packed store and the recent FIFO get all the capacity those
        steps need (nothing reallocates inside the graph), the FIFO is
        compacted, and the state at step 0 is recorded.  The kernels derive
        each step's state from it and the device step counter."""
        if self.quantize:
            self.reserve(self.n_q + max_steps + self.flush)
        need = self._rn + max_steps + 1
        if self._rbuf is None or self._r0 + need > self._rbuf.shape[2] or self._r0:
            buf = torch.empty((self.B, self.H, max(need, self._rbuf.shape[2] if self._rbuf is not None else 0),
                               self.D), dtype=self.dtype, device=self.device)
            if self._rn:
                buf[:, :, :self._rn].copy_(self.recent)
            self._rbuf, self._r0 = buf, 0
        self._g0 = (self.n_q, self._rn, self._r0)
        self._g_max = max_steps
        self._g_args = _lib.AppendArgs()
        self._g_args.struct_size = C.sizeof(_lib.AppendArgs)

    def append_graph(self, x: torch.Tensor, step: torch.Tensor):
        """The decode append of one token x [B, H, 1, D] in graph mode: one
        launch of innerq_append_step, state taken from the step counter."""
        a = self._g_args
        nq0, rn0, r00 = self._g0
        a.dtype, a.B, a.H, a.D = dtype_code(self.dtype), self.B, self.H, self.D
        a.x, a.x_sb, a.x_sh = x.data_ptr(), x.stride(0), x.stride(1)
        rb = self._rbuf
        a.fifo = rb.data_ptr()
        a.f_sb, a.f_sh, a.f_st = rb.stride()[:3]
        a.fifo_cap = rb.shape[2]
        a.codes, a.scale, a.zero = _ptr(self.codes), _ptr(self.scale), _ptr(self.zero)
        a.cap_tiles = self.cap_tiles
        a.norm_f = self.norm_f.data_ptr() if (self.normalize and self.norm_f is not None) else None
        a.bits = self.bits if self.quantize else 16
        a.group, a.mode, a.role, a.over_token = self.group, self.mode, self.role, int(self.over_token)
        a.flush = self.flush
        a.n_q, a.n_recent, a.r0 = nq0, rn0, r00
        a.max_steps = self._g_max
        _lib.call("innerq_append_step", C.byref(a), step.data_ptr(), stream_ptr(self.device))

    def state_after(self, n_steps: int) -> tuple[int, int]:
        """(n_q, n_recent) after n_steps graph-mode steps (host arithmetic)."""
        nq0, rn0, _ = self._g0
        f = self.flush if self.quantize else 0
        k = min(n_steps, (rn0 + n_steps) // f) if f else 0
        return nq0 + f * k, rn0 + n_steps - f * k

    def graph_end(self, n_steps: int):
        """Bring the host-side state up to date after n_steps replayed steps.
        More steps than graph_begin reserved raise: the kernels stopped at the
        reservation (appends write nothing past it), so the cache no longer
        holds every token."""
        if n_steps > self._g_max:
            raise RuntimeError(f"{n_steps} graph-mode steps replayed, {self._g_max} reserved by "
                               "graph_begin: the steps past the reservation were not appended")
        nq0, rn0, r00 = self._g0
        f = self.flush if self.quantize else 0
        k = min(n_steps, (rn0 + n_steps) // f) if f else 0
        self.n_q, self._rn, self._r0 = nq0 + f * k, rn0 + n_steps - f * k, r00 + f * k
        self._g0 = None

    def fill_side(self, s: _lib.Side, graph: bool = False) -> _lib.Side:
        """Write this side's current geometry into a (reused) C struct; the
        recent-window pointer is computed without building a tensor view.
        graph=True: the step-0 state of graph mode (FIFO base, offset and
        flush size; the kernel advances it by the step counter)."""
        if graph:
            nq0, rn0, r00 = self._g0
            s.codes, s.scale, s.zero = _ptr(self.codes), _ptr(self.scale), _ptr(self.zero)
            s.cap_tiles = self.cap_tiles
            if self.sink is not None and self.sink.shape[2]:
                s.sink = self.sink.data_ptr()
                s.sink_sb, s.sink_sh, s.sink_st = self.sink.stride()[:3]
                s.n_sink = self.sink.shape[2]
            else:
                s.sink, s.n_sink = None, 0
            rb = self._rbuf
            s.recent = rb.data_ptr()
            s.rec_sb, s.rec_sh, s.rec_st = rb.stride()[:3]
            s.n_q, s.n_recent, s.r0 = nq0, rn0, r00
            s.max_steps = self._g_max
            s.flush = self.flush if self.quantize else 0
            s.bits, s.group, s.mode, s.over_token = self.bits, self.group, self.mode, int(self.over_token)
            return s
        s.r0, s.flush, s.max_steps = 0, 0, 0
        s.codes2 = s.scale2 = s.zero2 = s.mask = None
        s.cap_tiles2 = 0
        nq = self.n_q
        s.codes = self.codes.data_ptr() if nq else None
        s.scale = self.scale.data_ptr() if nq else None
        s.zero = self.zero.data_ptr() if (nq and self.zero is not None) else None
        s.cap_tiles = self.cap_tiles
        if self.sink is not None and self.sink.shape[2]:
            s.sink = self.sink.data_ptr()
            s.sink_sb, s.sink_sh, s.sink_st = self.sink.stride()[:3]
            s.n_sink = self.sink.shape[2]
        else:
            s.sink, s.n_sink = None, 0
        if self._rn:
            rb = self._rbuf
            sb, sh, st, _ = rb.stride()
            s.recent = rb.data_ptr() + self._r0 * st * rb.element_size()
            s.rec_sb, s.rec_sh, s.rec_st = sb, sh, st
        else:
            s.recent = None
        s.n_q, s.n_recent = nq, self._rn
        s.bits, s.group, s.mode, s.over_token = self.bits, self.group, self.mode, int(self.over_token)
        return s

    def side_struct(self) -> _lib.Side:
        return self.fill_side(_lib.Side())


class HybridSide(PackedSide):
    """Hybrid mode (``quant.py:133-176``): every group is quantized twice —
    symmetric at ``bits`` (kept in this store) and asymmetric at ``bits - 1``
    (kept in ``self.zp``) — and a per-group mask chooses the symmetric one
    where its fp32 L1 error is lower.  Materialised through the dequant
    kernels, or, for values grouped over tokens, read by the fused attention
    kernel directly: ``self.mask_bits`` keeps the mask on the device as one
    bit per (group, dim), 16 bytes per group, bit ``col_scale_idx(dim)`` (the
    dims' order in the value scales) set where the group keeps its symmetric
    codes.

    The mask is computed from the GPU dequantization with torch sums, so on an
    exact tie of the two fp32 error sums (summation order differs from the
    reference's CPU sum) the choice can differ; both choices are valid
    reconstructions of that group."""

    def __init__(self, role, bits, group, over_token, w_sink, w_recent, flush, normalize=False):
        super().__init__(role, bits, group, _lib.SYM, over_token, w_sink, w_recent, flush, normalize)
        self.zp = PackedSide(role, bits - 1, group, _lib.ASYM, over_token, 0, 0, flush)
        self.masks = []
        self.mask_bits = None  # [B, H, groups of zp's capacity, 16] uint8

    @property
    def fusable(self) -> bool:
        return not self.quantize or (self.role == _lib.ROLE_V and self.over_token)

    # dims in the order of the value scales: bit (2 * (d >> 4) + ((d >> 3) & 1))
    # of 16-bit word d & 7 of a group's mask
    def _store_mask_bits(self, m: torch.Tensor, g0: int):
        """Pack the bool mask m [B, H, n_groups, D] of the groups from g0 on."""
        B, H, n, D = m.shape
        cap_groups = self.zp.cap_tiles * 32 // self.group
        if self.mask_bits is None or self.mask_bits.shape[2] < cap_groups:
            buf = torch.zeros((B, H, cap_groups, 16), dtype=torch.uint8, device=m.device)
            if self.mask_bits is not None:
                buf[:, :, :self.mask_bits.shape[2]].copy_(self.mask_bits)
            self.mask_bits = buf
        # d = mt*16 + h*8 + gid -> [gid][mt][h], 16 bits per gid
        bits = m.view(B, H, n, 8, 2, 8).permute(0, 1, 2, 5, 3, 4).reshape(B, H, n, 8, 16)
        w = (bits.to(torch.int32) << torch.arange(16, device=m.device, dtype=torch.int32)).sum(-1)
        by = torch.stack([(w & 0xFF), (w >> 8) & 0xFF], dim=-1).to(torch.uint8)  # little-endian words
        self.mask_bits[:, :, g0:g0 + n] = by.view(B, H, n, 16)

    def _check_supported(self):
        super()._check_supported()
        for k in ("dtype", "device", "B", "H", "D"):
            setattr(self.zp, k, getattr(self, k))
        self.zp._check_supported()

    def _quantize(self, x: torch.Tensor):
        if x.shape[2] == 0:
            return
        from . import quant as Q
        xs = x
        if self.normalize:
            raise NotImplementedError("hybrid mode with key normalisation")
        axis = 2 if self.over_token else 3
        qa = Q.quantize_asym(xs, self.group, self.bits - 1, axis)
        qs = Q.quantize_sym(xs, self.group, self.bits, axis)
        if self.over_token:
            da = Q.dequantize_tokendim_asym(*qa, self.group)
            ds = Q.dequantize_tokendim_sym(*qs, self.group)
            shp = (x.shape[0], x.shape[1], x.shape[2] // self.group, self.group, x.shape[3])
            red = 3
        else:
            da = Q.dequantize_channeldim_asym(*qa, self.group)
            ds = Q.dequantize_channeldim_sym(*qs, self.group)
            shp = (x.shape[0], x.shape[1], x.shape[2], x.shape[3] // self.group, self.group)
            red = 4
        xf = x.float()
        err_a = (da - xf).view(shp).abs().sum(red)
        err_s = (ds - xf).view(shp).abs().sum(red)
        m = err_a > err_s
        self.masks.append(m)
        g0 = self.n_q // self.group
        self.zp._quantize(x)
        PackedSide._quantize(self, x)
        if self.over_token:
            self._store_mask_bits(m, g0)

    def mask(self):
        return torch.cat(self.masks, dim=2) if self.masks else None

    def state_dict(self) -> dict:
        """The symmetric set (PackedSide.state_dict), the asymmetric set and
        the per-group masks."""
        d = super().state_dict()
        d["zp"] = self.zp.state_dict()
        m = self.mask()
        d["mask"] = None if m is None else m.cpu()
        return d

    def load_state_dict(self, d: dict, device) -> None:
        super().load_state_dict(d, device)
        self.zp.load_state_dict(d["zp"], device)
        self.masks, self.mask_bits = [], None
        if d["mask"] is not None:
            m = d["mask"].to(self.device)
            self.masks = [m]
            if self.over_token:
                self._store_mask_bits(m, 0)

    def materialize(self) -> torch.Tensor:
        out = super().materialize()
        if self.n_q == 0:
            return out
        ns, nq = self.n_sink, self.n_q
        zp_mid = torch.empty((self.B, self.H, nq, self.D), dtype=self.dtype, device=self.device)
        _lib.call("innerq_dequant", self.zp.codes.data_ptr(), self.zp.scale.data_ptr(),
                  self.zp.zero.data_ptr(), dtype_code(self.dtype), self.B, self.H, 0, nq, self.D,
                  self.zp.bits, self.group, _lib.ASYM, self.role, int(self.over_token),
                  self.zp.cap_tiles, None, zp_mid.data_ptr(), zp_mid.stride(0), zp_mid.stride(1),
                  zp_mid.stride(2), stream_ptr(self.device))
        m = self.mask()
        m = m.repeat_interleave(self.group, dim=2 if self.over_token else 3)
        mid = out[:, :, ns:ns + nq]
        mid.copy_(torch.where(m, mid, zp_mid))
        return out

    def fill_side(self, s: _lib.Side, graph: bool = False) -> _lib.Side:
        """The symmetric set as the side's store, plus the asymmetric set and
        the mask (mode INNERQ_HYBRID) once something is packed."""
        if graph:
            raise NotImplementedError("graph mode does not cover hybrid stores")
        super().fill_side(s)
        if self.n_q:
            zp = self.zp
            s.mode = _lib.HYBRID
            s.codes2, s.scale2, s.zero2 = zp.codes.data_ptr(), zp.scale.data_ptr(), zp.zero.data_ptr()
            s.mask, s.cap_tiles2 = self.mask_bits.data_ptr(), zp.cap_tiles
        else:
            s.codes2 = s.scale2 = s.zero2 = s.mask = None
            s.cap_tiles2 = 0
        return s

    def ref_views(self):
        if self.n_q == 0:
            return None, None, None
        cs, ss, sg = super().ref_views()
        ca, sa, za = self.zp.ref_views()
        return ({'zp': ca, 'nozp': cs}, {'zp': sa, 'nozp': ss, 'mask': self.mask()},
                {'zp': za, 'nozp': sg})
