"""Host-side mirror of the reference MoE interface over libmiag.

Names follow the reference engine (nextocodeoficial/motorIa):

  MoEEngine.moe(x, layer)   <- static int moe(mia_model*, dims, int layer)
                               (src/model/forward.c:167-197), batched over tokens
  MoEEngine.load_experts    <- the mia_expert_loader port
                               (include/mia/expert_cache.h:8) filling HBM once
  quantize_row_q8           <- mia_quantize_row_q8 (include/mia/quant.h:18)
  matvec                    <- mia_matvec (include/mia/matmul.h:11-12)

Errors surface as MiagError carrying the library's message, the way the
reference returns -1 with text in an err buffer.  There is no CPU path.
"""

from __future__ import annotations

import ctypes as C

import numpy as np

from . import _native as N
from .synth import Shape

MIA_F32, MIA_Q8_0 = 0, 1
PREFILL_MMA, PREFILL_TCGEN05 = 0, 1  # MIAG_PREFILL_* of miag.h


def _shape(shape: Shape, n_layers: int) -> N.Shape:
    return N.Shape(shape.dim, n_layers, shape.n_experts, shape.n_active, shape.expert_hidden,
                   shape.norm_topk, shape.norm_eps)


def blob_bytes(shape: Shape) -> int:
    s = _shape(shape, 1)
    return int(N.lib().miag_blob_bytes(C.byref(s)))


class MoEEngine:
    """One libmiag context: HBM-resident experts for n_layers MoE layers."""

    def __init__(self, shape: Shape, n_layers: int = 1, device: int = 0):
        self.shape = shape
        self.n_layers = n_layers
        self._lib = N.lib()
        self._ctx = C.c_void_p()
        s = _shape(shape, n_layers)
        err = N.errbuf()
        N.check(self._lib.miag_open(C.byref(self._ctx), C.byref(s), device, err, len(err)), err,
                "miag_open")

    @property
    def handle(self) -> int:
        return self._ctx.value

    def close(self) -> None:
        if self._ctx:
            self._lib.miag_close(self._ctx)
            self._ctx = C.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_layer(self, layer: int, ffn_norm: np.ndarray, router: np.ndarray,
                  bias: np.ndarray | None = None) -> None:
        fn = np.ascontiguousarray(ffn_norm, dtype=np.float32)
        rt = np.ascontiguousarray(router, dtype=np.float32)
        bs = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        err = N.errbuf()
        rc = self._lib.miag_set_layer(self._ctx, layer, fn.ctypes.data, rt.ctypes.data,
                                      None if bs is None else bs.ctypes.data, err, len(err))
        N.check(rc, err, "miag_set_layer")

    def upload_experts(self, layer: int, blobs: np.ndarray, first: int = 0) -> None:
        b = np.ascontiguousarray(blobs, dtype=np.uint8)
        if b.ndim != 2:
            raise ValueError("blobs must be [n_experts][blob_stride] uint8")
        err = N.errbuf()
        rc = self._lib.miag_upload_experts(self._ctx, layer, first, b.shape[0], b.ctypes.data,
                                           b.shape[1], err, len(err))
        N.check(rc, err, "miag_upload_experts")

    def load_experts(self, loader) -> None:
        """loader(layer, expert, dst: memoryview) -> int (0 = ok), the reference port."""
        nbytes = blob_bytes(self.shape)

        def tramp(_ctx, layer, expert, dst):
            view = (C.c_uint8 * nbytes).from_address(dst)
            try:
                return int(loader(layer, expert, memoryview(view).cast("B")))
            except Exception:
                return -1

        cb = N.LOADER(tramp)
        err = N.errbuf()
        rc = self._lib.miag_load_experts(self._ctx, cb, None, err, len(err))
        N.check(rc, err, "miag_load_experts")

    def load_layer(self, layer: int, lay) -> None:
        """Uploads a synth.Layer (dense tensors + expert blobs)."""
        self.set_layer(layer, lay.ffn_norm, lay.router, lay.bias)
        self.upload_experts(layer, lay.blobs)

    def moe(self, x: np.ndarray, layer: int = 0) -> np.ndarray:
        """Returns x + MoE(x) for x [T][dim] f32 (host in, host out)."""
        out = np.array(x, dtype=np.float32, order="C", copy=True)
        if out.ndim == 1:
            out = out[None, :]
        err = N.errbuf()
        rc = self._lib.miag_moe(self._ctx, layer, out.ctypes.data, out.shape[0], err, len(err))
        N.check(rc, err, "miag_moe")
        return out.reshape(np.shape(x))

    def moe_inplace(self, x: np.ndarray, layer: int = 0) -> None:
        """x += MoE(x) on a C-contiguous f32 host array (pinned or not), in place."""
        if x.dtype != np.float32 or not x.flags["C_CONTIGUOUS"] or x.ndim != 2:
            raise ValueError("x must be a C-contiguous float32 [T][dim] array")
        err = N.errbuf()
        rc = self._lib.miag_moe(self._ctx, layer, x.ctypes.data, x.shape[0], err, len(err))
        N.check(rc, err, "miag_moe")

    def moe_device(self, x_ptr: int, n_tokens: int, layer: int = 0, stream: int | None = None):
        """Enqueues the block on a device buffer x_ptr [n_tokens][dim] (in place)."""
        err = N.errbuf()
        rc = self._lib.miag_moe_async(self._ctx, layer, C.c_void_p(x_ptr), n_tokens,
                                      C.c_void_p(stream or 0), err, len(err))
        N.check(rc, err, "miag_moe_async")

    # -- the block in three device steps (expert parallelism; see ep.py)
    def dx_stride(self) -> int:
        """f32 block scales per row of the dx buffers of route/experts."""
        return int(self._lib.miag_dx_stride(C.byref(_shape(self.shape, 1))))

    def route_device(self, x_ptr: int, n_tokens: int, idx_ptr: int, w_ptr: int, xq_ptr: int,
                     dx_ptr: int, layer: int = 0, stream: int | None = None) -> None:
        """Enqueues the router on x [n][dim]: idx, w [n][K]; xq [n][dim] int8 and
        dx [n][dx_stride] f32, the Q8_0 form of the normalised rows."""
        err = N.errbuf()
        rc = self._lib.miag_route_async(self._ctx, layer, C.c_void_p(x_ptr), n_tokens,
                                        C.c_void_p(idx_ptr), C.c_void_p(w_ptr),
                                        C.c_void_p(xq_ptr), C.c_void_p(dx_ptr),
                                        C.c_void_p(stream or 0), err, len(err))
        N.check(rc, err, "miag_route_async")

    def experts_device(self, xq_ptr: int, dx_ptr: int, n_rows: int, pair_row_ptr: int,
                       pair_expert_ptr: int, n_pairs: int, y_ptr: int, layer: int = 0,
                       stream: int | None = None) -> None:
        """Enqueues the expert products of n_pairs (row, expert) pairs: y [n_pairs][dim]
        in pair order."""
        err = N.errbuf()
        rc = self._lib.miag_experts_async(self._ctx, layer, C.c_void_p(xq_ptr),
                                          C.c_void_p(dx_ptr), n_rows, C.c_void_p(pair_row_ptr),
                                          C.c_void_p(pair_expert_ptr), n_pairs,
                                          C.c_void_p(y_ptr), C.c_void_p(stream or 0), err,
                                          len(err))
        N.check(rc, err, "miag_experts_async")

    def combine_device(self, x_ptr: int, n_tokens: int, w_ptr: int, y_ptr: int,
                       y_pos_ptr: int = 0, stream: int | None = None) -> None:
        """Enqueues x[t] += sum_j w[t][j] * y[row(t*K + j)], j in order; row(p) =
        y_pos[p], or p without y_pos."""
        err = N.errbuf()
        rc = self._lib.miag_combine_async(self._ctx, C.c_void_p(x_ptr), n_tokens,
                                          C.c_void_p(w_ptr), C.c_void_p(y_ptr),
                                          C.c_void_p(y_pos_ptr or 0), C.c_void_p(stream or 0),
                                          err, len(err))
        N.check(rc, err, "miag_combine_async")

    def ep_plan_device(self, idx_ptr: int, n_tokens: int, n_ranks: int, experts_per_rank: int,
                       strided: bool, counts_ptr: int, send_rows_ptr: int, pair_meta_ptr: int,
                       y_pos_ptr: int, stream: int | None = None) -> None:
        """Enqueues the expert-parallel dispatch plan of idx [n][K]: counts
        [G][2] int64 (rows, pairs) per rank, send_rows [n*G], pair_meta
        [n*K][2], y_pos [n*K] (miag_ep_plan_async)."""
        err = N.errbuf()
        rc = self._lib.miag_ep_plan_async(self._ctx, C.c_void_p(idx_ptr), n_tokens, n_ranks,
                                          experts_per_rank, int(strided), C.c_void_p(counts_ptr),
                                          C.c_void_p(send_rows_ptr), C.c_void_p(pair_meta_ptr),
                                          C.c_void_p(y_pos_ptr), C.c_void_p(stream or 0), err,
                                          len(err))
        N.check(rc, err, "miag_ep_plan_async")

    def ep_pack_device(self, xq_ptr: int, dx_ptr: int, send_rows_ptr: int, n_rows: int,
                       pair_meta_ptr: int, n_pairs: int, all_counts_ptr: int, rank: int,
                       n_ranks: int, rec_ptr: int, meta_out_ptr: int,
                       stream: int | None = None) -> None:
        """Enqueues the send records of rank `rank` (miag_ep_pack_async)."""
        err = N.errbuf()
        rc = self._lib.miag_ep_pack_async(self._ctx, C.c_void_p(xq_ptr), C.c_void_p(dx_ptr),
                                          C.c_void_p(send_rows_ptr), n_rows,
                                          C.c_void_p(pair_meta_ptr), n_pairs,
                                          C.c_void_p(all_counts_ptr), rank, n_ranks,
                                          C.c_void_p(rec_ptr), C.c_void_p(meta_out_ptr),
                                          C.c_void_p(stream or 0), err, len(err))
        N.check(rc, err, "miag_ep_pack_async")

    def ep_buffer(self, y_rows: int) -> tuple[int, int, bytes]:
        """This rank's exchange buffer for y_rows rows (grown when needed):
        (rows address, flags address, IPC handle bytes) (miag_ep_buffer)."""
        y, fl, h = C.c_void_p(), C.c_void_p(), C.create_string_buffer(64)
        err = N.errbuf()
        rc = self._lib.miag_ep_buffer(self._ctx, y_rows, C.byref(y), C.byref(fl), h, err, len(err))
        N.check(rc, err, "miag_ep_buffer")
        return int(y.value), int(fl.value), bytes(h.raw)

    def ep_open_peer(self, handle: bytes) -> tuple[int, int]:
        """Maps a peer's exchange buffer: (rows address, flags address)."""
        y, fl = C.c_void_p(), C.c_void_p()
        err = N.errbuf()
        rc = self._lib.miag_ep_open_peer(self._ctx, C.c_char_p(handle), C.byref(y), C.byref(fl),
                                         err, len(err))
        N.check(rc, err, "miag_ep_open_peer")
        return int(y.value), int(fl.value)

    def ep_close_peers(self) -> None:
        err = N.errbuf()
        N.check(self._lib.miag_ep_close_peers(self._ctx, err, len(err)), err, "miag_ep_close_peers")

    def experts_to_ranks_device(self, xq_ptr: int, dx_ptr: int, n_rows: int, pair_row_ptr: int,
                                pair_expert_ptr: int, n_pairs: int, rank: int, src_end, dst,
                                flags, seq: int, layer: int = 0,
                                stream: int | None = None) -> None:
        """Expert products whose y rows go to the pairs' origin ranks
        (miag_experts_to_ranks_async); src_end, dst, flags: one per rank."""
        G = len(src_end)
        ends = (C.c_int32 * G)(*src_end)
        dsts = (C.c_void_p * G)(*dst)
        fls = (C.c_void_p * G)(*flags)
        err = N.errbuf()
        rc = self._lib.miag_experts_to_ranks_async(
            self._ctx, layer, C.c_void_p(xq_ptr), C.c_void_p(dx_ptr), n_rows,
            C.c_void_p(pair_row_ptr), C.c_void_p(pair_expert_ptr), n_pairs, G, rank, ends, dsts,
            fls, seq, C.c_void_p(stream or 0), err, len(err))
        N.check(rc, err, "miag_experts_to_ranks_async")

    def ep_wait_device(self, flags_ptr: int, n_ranks: int, seq: int,
                       stream: int | None = None) -> None:
        """Enqueues the wait for every rank's flag here to reach seq."""
        err = N.errbuf()
        rc = self._lib.miag_ep_wait_async(self._ctx, C.c_void_p(flags_ptr), n_ranks, seq,
                                          C.c_void_p(stream or 0), err, len(err))
        N.check(rc, err, "miag_ep_wait_async")

    def sync(self, stream: int | None = None) -> None:
        err = N.errbuf()
        N.check(self._lib.miag_sync(self._ctx, C.c_void_p(stream or 0), err, len(err)), err,
                "miag_sync")

    def selftest_wait_timeout(self, timeout_us: int = 2000) -> str:
        """Runs the library's bounded wait on a barrier that never completes;
        returns the error text it reported ('' if it did not report)."""
        err = N.errbuf()
        rc = self._lib.miag_selftest_wait_timeout(self._ctx, timeout_us, err, len(err))
        return err.value.decode(errors="replace") if rc != 0 else ""

    def routing(self, n_tokens: int) -> dict:
        """Routing of the last call: idx, w [T][K]; counts [E]; offsets [E+1]; perm [T*K]."""
        K, E = self.shape.n_active, self.shape.n_experts
        idx = np.zeros((n_tokens, K), np.int32)
        w = np.zeros((n_tokens, K), np.float32)
        counts = np.zeros(E, np.int32)
        offsets = np.zeros(E + 1, np.int32)
        perm = np.zeros(n_tokens * K, np.int32)
        err = N.errbuf()
        rc = self._lib.miag_routing(self._ctx, idx.ctypes.data, w.ctypes.data, counts.ctypes.data,
                                    offsets.ctypes.data, perm.ctypes.data, err, len(err))
        N.check(rc, err, "miag_routing")
        return dict(idx=idx, w=w, counts=counts, offsets=offsets, perm=perm)

    def router_logits(self, n_tokens: int) -> np.ndarray:
        """Router logits (+ bias) [T][E] of the last call."""
        out = np.zeros((n_tokens, self.shape.n_experts), np.float32)
        err = N.errbuf()
        N.check(self._lib.miag_router_logits(self._ctx, out.ctypes.data, err, len(err)), err,
                "miag_router_logits")
        return out

    def last_launch_count(self) -> int:
        return int(self._lib.miag_last_launch_count(self._ctx))

    def set_prefill_kernel(self, kind: int) -> None:
        """PREFILL_TCGEN05 or PREFILL_MMA for prefill-size batches (same bits)."""
        err = N.errbuf()
        N.check(self._lib.miag_set_prefill_kernel(self._ctx, kind, err, len(err)), err,
                "miag_set_prefill_kernel")

    def set_transfer_chunks(self, chunks: int) -> None:
        """Pieces a host-API call of >= 2048 tokens moves through (1: one)."""
        if self._lib.miag_set_transfer_chunks(self._ctx, int(chunks)) != 0:
            raise N.MiagError(f"miag_set_transfer_chunks: bad count {chunks}")

    def set_host_copy_threads(self, threads: int) -> None:
        """Host threads that copy a pageable buffer of >= 1 MiB through the
        context's pinned staging buffer (0: the driver's pageable copies)."""
        if self._lib.miag_set_host_copy_threads(self._ctx, int(threads)) != 0:
            raise N.MiagError(f"miag_set_host_copy_threads: bad count {threads}")

    def prefill_kernel(self) -> int:
        return int(self._lib.miag_prefill_kernel(self._ctx))

    def profile(self, enable: bool = True) -> None:
        """Brackets every kernel stage of later calls with CUDA events."""
        self._lib.miag_profile(self._ctx, int(enable))

    def profile_read(self) -> dict:
        """{stage: (milliseconds, launches)} since the last read."""
        n = self._lib.miag_profile_stages()
        ms = np.zeros(n, np.float64)
        launches = np.zeros(n, np.int32)
        err = N.errbuf()
        N.check(self._lib.miag_profile_read(self._ctx, ms.ctypes.data, launches.ctypes.data, err,
                                            len(err)), err, "miag_profile_read")
        return {self._lib.miag_profile_stage_name(i).decode(): (float(ms[i]), int(launches[i]))
                for i in range(n)}


def quantize_row_q8(x_ptr: int, y_ptr: int, n: int, stream: int | None = None) -> None:
    """Device mia_quantize_row_q8: x f32 [n] -> y n/32 36-byte blocks."""
    rc = N.lib().miag_quantize_row_q8(C.c_void_p(x_ptr), C.c_void_p(y_ptr), n,
                                      C.c_void_p(stream or 0))
    if rc:
        raise N.MiagError("miag_quantize_row_q8 failed")


def matvec(out_ptr: int, w_ptr: int, wtype: int, x_ptr: int, xq_ptr: int, rows: int, cols: int,
           stream: int | None = None) -> None:
    """Device mia_matvec (f32 or Q8_0 rows)."""
    rc = N.lib().miag_matvec(C.c_void_p(out_ptr), C.c_void_p(w_ptr), wtype, C.c_void_p(x_ptr),
                             C.c_void_p(xq_ptr), rows, cols, C.c_void_p(stream or 0))
    if rc:
        raise N.MiagError("miag_matvec failed")
