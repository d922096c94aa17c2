"""Python host side of the B200 quantized weight-streaming path.

A thin ctypes layer over the C ABI in include/pulsar_b200.h (built as
pulsar-asm_b200/lib/libpulsar_b200.so). Device buffers are torch CUDA tensors
(PyTorch is used for device memory and streams only); every computation runs in
the library's own sm_100a kernels. There is no CPU fallback: if the library is
missing, importing the wrapper classes raises.

The interface mirrors the reference engine's entry points:
  Q8Tensor.gemv      <- gemv() / gemv_f()      lfm3_nanode.cu:1916-1966, :3634-3664
  Q8Tensor.gemm      <- pf_gemv_T()            lfm3_nanode.cu:4840-4968
  Q1Tensor.gemv      <- pq1 GEMV launchers     pq1_swar_sm53.cu:1129-1175
  Model.open         <- load_blob()            lfm3_nanode.cu:1404-1733
  Model.layer_step   <- layer_body()           lfm3_nanode.cu:3739-3856
  Model.decode_token <- the step loop's token  lfm3_nanode.cu:5828-6300
"""
import ctypes as C
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
LIB_PATH = os.path.join(PKG, "lib", "libpulsar_b200.so")
HEADER = os.path.join(os.path.dirname(PKG), "include", "pulsar_b200.h")

PB_OK = 0
PB_DT_BF16, PB_DT_F32, PB_DT_F16 = 0, 1, 2
ERRORS = {-1: "PB_EINVAL", -2: "PB_ENOMEM", -3: "PB_ECUDA", -4: "PB_EIO", -5: "PB_ECRC",
          -6: "PB_EFORMAT", -8: "PB_ENOTSUP"}

_lib = None


class PBError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__("%s (%d): %s" % (ERRORS.get(code, "?"), code, msg))
        self.code = code


def build(force=False):
    """Compile the CUDA library in-tree (sm_100a)."""
    args = ["make", "-s", "-C", PKG]
    if force:
        subprocess.check_call(["make", "-s", "-C", PKG, "clean"])
    subprocess.check_call(args)


class _Info(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("hidden", "inter", "n_layers", "n_heads", "n_kv",
                                       "head_dim", "vocab", "conv_w", "n_attn",
                                       "sliding_window")] + \
               [(n, C.c_float) for n in ("rope_theta", "rope_partial", "norm_eps")] + \
               [("weight_bytes", C.c_uint64)]


def lib():
    """Load libpulsar_b200.so (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise OSError("libpulsar_b200.so not built (%s); run pulsar_b200.build()" % LIB_PATH)
    L = C.CDLL(LIB_PATH)
    vp, i, u64, sz = C.c_void_p, C.c_int, C.c_uint64, C.c_size_t
    pvp = C.POINTER(C.c_void_p)
    L.pb_version.restype = i
    L.pb_last_error.argtypes = [C.c_char_p, sz]
    L.pb_launch_count.restype = u64
    L.pb_q8_pack.argtypes = [vp, vp, i, i, i, i, vp, pvp]
    L.pb_q8_free.argtypes = [vp]
    L.pb_q8_shape.argtypes = [vp, C.POINTER(i), C.POINTER(i)]
    L.pb_q8_gemv.argtypes = [vp, vp, vp, i, vp]
    L.pb_q8_gemm.argtypes = [vp, i, vp, vp, i, vp]
    L.pb_q80_quantize.argtypes = [vp, i, vp, vp, vp]
    L.pb_q80_gemv.argtypes = [vp, vp, vp, vp, vp, vp]
    L.pb_q80tc_pack.argtypes = [vp, vp, i, i, i, i, vp, pvp]
    L.pb_bf16_relayout.argtypes = [vp, vp, i, i, vp]
    L.pb_bf16_gemv.argtypes = [vp, i, i, vp, vp, vp]
    L.pb_q80_gemm.argtypes = [vp, i, vp, vp, vp, vp, vp]
    L.pb_q80_gemm_status.argtypes = [vp]
    L.pb_q1_pack.argtypes = [vp, i, i, i, vp, pvp]
    L.pb_q1_free.argtypes = [vp]
    L.pb_q8k_quantize.argtypes = [vp, i, vp, vp]
    L.pb_qlow_pack.argtypes = [vp, vp, i, i, i, i, vp, pvp]
    L.pb_qlow_free.argtypes = [vp]
    L.pb_qlow_gemv.argtypes = [vp, vp, vp, vp]
    L.pb_qlow_gemm.argtypes = [vp, i, vp, vp, vp]
    L.pb_qlow_status.argtypes = [vp, vp]
    L.pb_tq_scratch_bytes.argtypes = [i, i]
    L.pb_tq_scratch_bytes.restype = C.c_longlong
    L.pb_tq_store.argtypes = [i, vp, i, vp, vp, vp, vp, i, i, vp]
    L.pb_tq_attention.argtypes = [i, vp, vp, vp, vp, vp, i, i, i, vp, vp, vp]
    L.pb_sample_topkpp.argtypes = [vp, i, i, C.c_longlong, C.c_float, C.c_float, i, C.c_float, vp, vp, vp]
    L.pb_q1_gemv.argtypes = [vp, vp, vp, vp, vp]
    L.pq1_pq1_compat_gemv.restype = None
    L.pq1_pq1_compat_gemv.argtypes = [i, i, vp, vp, vp, vp]
    L.pq1_pq1_compat_gemv_batch.argtypes = [C.POINTER(vp), C.POINTER(i), i, i, C.POINTER(vp), vp]
    L.pb_open.argtypes = [C.c_char_p, i, pvp]
    L.pb_close.argtypes = [vp]
    L.pb_model_get_info.argtypes = [vp, C.POINTER(_Info)]
    L.pb_tensor_id.argtypes = [vp, C.c_char_p]
    L.pb_model_gemv.argtypes = [vp, i, vp, vp, vp]
    L.pb_state_create.argtypes = [vp, i, pvp]
    L.pb_state_destroy.argtypes = [vp]
    L.pb_state_reset.argtypes = [vp, vp]
    L.pb_layer_step.argtypes = [vp, vp, i, i, vp, vp]
    L.pb_decode_token.argtypes = [vp, vp, i, i, C.POINTER(i), vp, vp]
    L.pb_decode_greedy.argtypes = [vp, vp, i, i, i, vp, vp]
    L.pb_state_debug.argtypes = [vp, i, pvp, C.POINTER(sz)]
    L.pb_decode_prompt.argtypes = [vp, vp, vp, i, i, vp, vp]
    L.pb_decode_kernels_per_token.argtypes = [vp]
    L.pb_time_step_kernel.argtypes = [vp, vp, i, i, C.POINTER(C.c_float), C.POINTER(C.c_double), vp]
    L.pb_test_expf.argtypes = [vp, vp, i, vp]
    L.pb_test_grid_wait.argtypes = [vp, C.c_uint, C.c_uint, vp, vp]
    L.pb_layer_step_noalloc.argtypes = [vp, vp, i, i, vp, vp]
    L.pb_state_status.argtypes = [vp, vp]
    L.pb_prefill_chunk.argtypes = [vp, vp, vp, i, i, vp, vp, vp]
    L.pb_decode_batch.argtypes = [vp, C.POINTER(vp), i, vp, vp, vp, vp, vp]
    L.pb_nccl_unique_id.argtypes = [vp, sz]
    L.pb_state_shard.argtypes = [vp, i, i, vp]
    L.pb_bonsai_create.argtypes = [C.POINTER(BonsaiCfg), i, pvp]
    L.pb_bonsai_destroy.argtypes = [vp]
    L.pb_bonsai_set_q1.argtypes = [vp, i, i, vp, i, vp]
    L.pb_bonsai_set_norm.argtypes = [vp, i, i, vp, i, vp]
    L.pb_bonsai_state_create.argtypes = [vp, i, pvp]
    L.pb_bonsai_state_create_tq.argtypes = [vp, i, i, pvp]
    L.pb_bonsai_state_destroy.argtypes = [vp]
    L.pb_bonsai_state_kv.argtypes = [vp, i, i, pvp]
    L.pb_bonsai_state_residual.argtypes = [vp, vp, vp]
    L.pb_bonsai_state_fallbacks.argtypes = [vp, C.POINTER(i)]
    L.pb_bonsai_state_status.argtypes = [vp, vp]
    L.pb_bonsai_decode.argtypes = [vp, vp, i, i, vp, vp, C.POINTER(i), vp]
    L.pb_bonsai_decode_greedy.argtypes = [vp, vp, i, i, i, vp, vp]
    _lib = L
    return L


class BonsaiCfg(C.Structure):
    """pb_bonsai_cfg (include/pulsar_b200.h)"""
    _fields_ = [(n, C.c_int) for n in ("hidden", "inter", "n_layers", "n_heads", "n_kv", "vocab")] + \
               [("rope_factor", C.c_float), ("rope_orig_ctx", C.c_int), ("rope_base", C.c_float),
                ("attn_scale", C.c_float)]


def nccl_unique_id():
    """a fresh NCCL unique id (128 bytes) for State.shard"""
    b = C.create_string_buffer(128)
    check(lib().pb_nccl_unique_id(b, 128))
    return b.raw


def last_error():
    buf = C.create_string_buffer(512)
    lib().pb_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def check(rc):
    if rc != PB_OK:
        raise PBError(rc, last_error())
    return rc


def launch_count():
    return int(lib().pb_launch_count())


def _ptr(t):
    """device pointer of a torch tensor (or None)."""
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream(stream=None):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def _produced(t):
    """A CUDA tensor handed to an upload is read on the upload's stream, which
    need not be the stream that wrote it: wait until the tensor's producer (the
    current stream of its device) has finished. Uploads are one-time setup."""
    import torch
    if isinstance(t, torch.Tensor) and t.is_cuda:
        torch.cuda.current_stream(t.device).synchronize()


class Q8Tensor:
    """A packed Q8 weight matrix on the device (int8 codes + per-32 scales)."""

    def __init__(self, codes, scales, stream=None, tensor_cores=False):
        """codes: int8 [N, K]; scales: fp16 (Q8_0) or fp32 (.lfm3q8 dtype 1)
        [N, K/32]; torch CUDA tensors or numpy arrays (host). tensor_cores:
        pack for the integer GEMM on the tensor cores (gemm_int) instead of the
        streaming GEMV layout."""
        import torch
        L = lib()
        N, K = codes.shape
        if isinstance(codes, torch.Tensor):
            sdt = PB_DT_F32 if scales.dtype == torch.float32 else PB_DT_F16
            on_dev = 1 if codes.is_cuda else 0
            _produced(codes)
            _produced(scales)
            cp, sp = C.c_void_p(codes.data_ptr()), C.c_void_p(scales.data_ptr())
        else:
            import numpy as np
            sdt = PB_DT_F32 if scales.dtype == np.float32 else PB_DT_F16
            on_dev = 0
            codes = np.ascontiguousarray(codes)
            scales = np.ascontiguousarray(scales)
            cp, sp = codes.ctypes.data_as(C.c_void_p), scales.ctypes.data_as(C.c_void_p)
        h = C.c_void_p()
        pack = L.pb_q80tc_pack if tensor_cores else L.pb_q8_pack
        check(pack(cp, sp, sdt, N, K, on_dev, _stream(stream), C.byref(h)))
        self.h, self.N, self.K = h, N, K

    def gemv(self, x, y, stream=None):
        """x: bf16 [K] (device); y: bf16 or fp32 [N] (device)."""
        import torch
        dt = PB_DT_F32 if y.dtype == torch.float32 else PB_DT_BF16
        check(lib().pb_q8_gemv(self.h, _ptr(x), _ptr(y), dt, _stream(stream)))

    def gemm(self, x, y, stream=None):
        """x: bf16 [T, K]; y: bf16 or fp32 [T, N]."""
        import torch
        dt = PB_DT_F32 if y.dtype == torch.float32 else PB_DT_BF16
        check(lib().pb_q8_gemm(self.h, x.shape[0], _ptr(x), _ptr(y), dt, _stream(stream)))

    def gemv_int(self, qx, dx, y, isum=None, stream=None):
        check(lib().pb_q80_gemv(self.h, _ptr(qx), _ptr(dx), _ptr(y), _ptr(isum), _stream(stream)))

    def gemm_int(self, qx, dx, y, isum=None, stream=None):
        """tensor-core integer GEMM: qx int8 [T, K], dx fp16 bits [T, K/32],
        y fp32 [T, N], isum (optional) int32 [T, N, K/32]"""
        check(lib().pb_q80_gemm(self.h, qx.shape[0], _ptr(qx), _ptr(dx), _ptr(y), _ptr(isum), _stream(stream)))

    @staticmethod
    def gemm_int_status(stream=None):
        check(lib().pb_q80_gemm_status(_stream(stream)))

    def __del__(self):
        try:
            if self.h:
                lib().pb_q8_free(self.h)
                self.h = None
        except Exception:
            pass


def q80_quantize(x, qx, dx, stream=None):
    """per 32-block Q8_0 quantisation of x (any shape, last dim % 32 == 0)"""
    check(lib().pb_q80_quantize(_ptr(x), x.numel(), _ptr(qx), _ptr(dx), _stream(stream)))


def q8k_quantize(x, xq, stream=None):
    check(lib().pb_q8k_quantize(_ptr(x), x.shape[0], _ptr(xq), _stream(stream)))


class QlowTensor:
    """A Q4 / Q5 matrix (blob dtypes 6 / 7, the exporter's tiled payload) on
    the device; gemv / gemm take and give bf16 bits (int16 tensors)."""

    def __init__(self, codes, scales, bits, N, K, stream=None):
        self.N, self.K, self.bits = N, K, bits
        h = C.c_void_p()
        on_dev = hasattr(codes, "is_cuda") and codes.is_cuda
        if on_dev:
            _produced(codes)
            _produced(scales)
            cp, sp = _ptr(codes), _ptr(scales)
        else:
            import numpy as np
            codes = np.ascontiguousarray(codes, np.uint8)
            scales = np.ascontiguousarray(scales, np.uint16)
            cp, sp = codes.ctypes.data, scales.ctypes.data
        check(lib().pb_qlow_pack(cp, sp, bits, N, K, 1 if on_dev else 0, _stream(stream), C.byref(h)))
        self.h = h

    def gemv(self, x, y, stream=None):
        check(lib().pb_qlow_gemv(self.h, _ptr(x), _ptr(y), _stream(stream)))

    def gemm(self, x, y, stream=None):
        check(lib().pb_qlow_gemm(self.h, x.shape[0], _ptr(x), _ptr(y), _stream(stream)))

    def status(self, stream=None):
        check(lib().pb_qlow_status(self.h, _stream(stream)))

    def __del__(self):
        try:
            if self.h:
                lib().pb_qlow_free(self.h)
                self.h = None
        except Exception:
            pass


def tq_store(bits, rows, npos, kcode, kscale, vcode, vscale, nkv, ctx, stream=None):
    """TurboQuant encode of rows (f16 bits [2 nkv][128]) at position npos"""
    check(lib().pb_tq_store(int(bits), _ptr(rows), int(npos), _ptr(kcode), _ptr(kscale), _ptr(vcode), _ptr(vscale),
                            int(nkv), int(ctx), _stream(stream)))


def tq_attention(bits, q, kcode, kscale, vcode, vscale, nkv, ctx, T, atto, scratch=None, stream=None):
    """attention of q (fp32 [4 nkv][128]) over positions 0..T-1 of a TurboQuant cache"""
    import torch
    if scratch is None:
        scratch = torch.empty(int(lib().pb_tq_scratch_bytes(nkv, ctx)) // 4, dtype=torch.float32, device=q.device)
    check(lib().pb_tq_attention(int(bits), _ptr(q), _ptr(kcode), _ptr(kscale), _ptr(vcode), _ptr(vscale), int(nkv),
                                int(ctx), int(T), _ptr(atto), _ptr(scratch), _stream(stream)))


def sample_topkpp(logits, temp, topp, topk, minp, rng, ids, stream=None):
    """fwd8.c's sampler on the device for every row of logits (fp32 [B][n]):
    top-k, min-p, top-p on the raw logits, temperature last, softmax draw;
    rng (uint64 as int64 [B]) holds each row's generator state and advances
    when temp > 0; ids (int32 [B]) receives the ids (-1 for a row with a NaN)"""
    lg = logits if logits.dim() == 2 else logits.view(1, -1)
    check(lib().pb_sample_topkpp(_ptr(lg), lg.shape[0], lg.shape[1], lg.stride(0), float(temp), float(topp),
                                 int(topk), float(minp), _ptr(rng) if rng is not None else None, _ptr(ids),
                                 _stream(stream)))


class Q1Tensor:
    """A packed Q1_0 matrix (18-byte blocks per 128 weights) on the device."""

    def __init__(self, blocks, rows, K, stream=None):
        import torch
        if isinstance(blocks, torch.Tensor):
            on_dev = 1 if blocks.is_cuda else 0
            _produced(blocks)
            bp = C.c_void_p(blocks.data_ptr())
        else:
            import numpy as np
            blocks = np.ascontiguousarray(blocks)
            on_dev = 0
            bp = blocks.ctypes.data_as(C.c_void_p)
        h = C.c_void_p()
        check(lib().pb_q1_pack(bp, rows, K, on_dev, _stream(stream), C.byref(h)))
        self.h, self.rows, self.K = h, rows, K

    def gemv(self, xq, y, isum=None, stream=None):
        check(lib().pb_q1_gemv(self.h, _ptr(xq), _ptr(y), _ptr(isum), _stream(stream)))

    def __del__(self):
        try:
            if self.h:
                lib().pb_q1_free(self.h)
                self.h = None
        except Exception:
            pass


def device_expf(x, y, stream=None):
    """test hook: the kernels' e^x on a device fp32 tensor."""
    check(lib().pb_test_expf(_ptr(x), _ptr(y), x.numel(), _stream(stream)))


def device_grid_wait(counter, target, limit, stream=None):
    """test hook: one bounded grid wait of the persistent decode kernel on a
    device int32 counter; 1 = gave up after `limit` polls, 2 = passed."""
    import torch
    status = torch.zeros(1, dtype=torch.int32, device=counter.device)
    check(lib().pb_test_grid_wait(_ptr(counter), target, limit, _ptr(status), _stream(stream)))
    torch.cuda.synchronize()
    return int(status.item())


def compat_gemv(rows, cols, w, xq, y):
    """pq1_pq1_compat_gemv on host numpy arrays (w: Q1_0 bytes, xq: Q8_K bytes)."""
    lib().pq1_pq1_compat_gemv(rows, cols, w.ctypes.data_as(C.c_void_p), None,
                              y.ctypes.data_as(C.c_void_p), xq.ctypes.data_as(C.c_void_p))


class Model:
    """An LFM3-style backbone loaded from an .lfm3q8 blob."""

    def __init__(self, path, device=0):
        h = C.c_void_p()
        check(lib().pb_open(path.encode(), device, C.byref(h)))
        self.h = h
        info = _Info()
        check(lib().pb_model_get_info(h, C.byref(info)))
        self.info = {k: getattr(info, k) for k, _ in _Info._fields_}

    def tensor_id(self, name):
        r = lib().pb_tensor_id(self.h, name.encode())
        if r < 0:
            raise PBError(r, last_error())
        return r

    def gemv(self, name, x, y, stream=None):
        """y (bf16 bits [N]) = the named matrix x (bf16 bits [K]); models holding
        Q4 / Q5 records (pb_model_gemv)"""
        check(lib().pb_model_gemv(self.h, self.tensor_id(name), _ptr(x), _ptr(y), _stream(stream)))

    def decode_batch(self, states, tokens, pos, ids, logits=None, stream=None):
        """one integer-path decode step of len(states) sequences: device int32
        tokens [B] and positions [B]; ids (device int32 [B]) receives the greedy ids"""
        arr = (C.c_void_p * len(states))(*[st.h.value if isinstance(st.h, C.c_void_p) else st.h for st in states])
        check(lib().pb_decode_batch(self.h, arr, len(states), _ptr(tokens), _ptr(pos), _ptr(ids), _ptr(logits),
                                    _stream(stream)))

    def new_state(self, max_ctx):
        return State(self, max_ctx)

    def close(self):
        if self.h:
            lib().pb_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class State:
    """KV cache (fp16), conv rings and per-sequence control block."""

    def __init__(self, model, max_ctx):
        h = C.c_void_p()
        check(lib().pb_state_create(model.h, max_ctx, C.byref(h)))
        self.h, self.model, self.max_ctx = h, model, max_ctx

    def reset(self, stream=None):
        check(lib().pb_state_reset(self.h, _stream(stream)))

    def layer_step(self, layer, pos, x, stream=None):
        check(lib().pb_layer_step(self.model.h, self.h, layer, pos, _ptr(x), _stream(stream)))

    def layer_step_noalloc(self, layer, pos, x, stream=None):
        """the layer step with its scratch in a static device array: for callers
        that cannot allocate device memory (same results as layer_step)."""
        check(lib().pb_layer_step_noalloc(self.model.h, self.h, layer, pos, _ptr(x), _stream(stream)))

    def decode_token(self, token, pos, logits=None, stream=None):
        out = C.c_int(-1)
        check(lib().pb_decode_token(self.model.h, self.h, int(token), int(pos), C.byref(out),
                                    _ptr(logits), _stream(stream)))
        return out.value

    def decode_token_async(self, token, pos, stream=None):
        check(lib().pb_decode_token(self.model.h, self.h, int(token), int(pos), None, None,
                                    _stream(stream)))

    def decode_greedy(self, token, pos0, n, ids, stream=None):
        check(lib().pb_decode_greedy(self.model.h, self.h, int(token), int(pos0), int(n),
                                     _ptr(ids), _stream(stream)))

    def decode_prompt(self, tokens, pos0, ids=None, stream=None):
        """tokens: device int32 [n]; ids (optional device int32 [n])."""
        check(lib().pb_decode_prompt(self.model.h, self.h, _ptr(tokens), tokens.numel(), int(pos0),
                                     _ptr(ids), _stream(stream)))

    def prefill_chunk(self, tokens, pos0, ids=None, logits=None, stream=None):
        """integer-path chunked prefill of device int32 tokens [T] at pos0.."""
        check(lib().pb_prefill_chunk(self.model.h, self.h, _ptr(tokens), tokens.shape[0], int(pos0), _ptr(ids),
                                     _ptr(logits), _stream(stream)))

    def status(self, stream=None):
        """synchronise and raise if the decode kernel recorded a failure."""
        check(lib().pb_state_status(self.h, _stream(stream)))

    def shard(self, rank, world, uid):
        """row-shard this state's decode over `world` ranks (collective);
        uid: the 128-byte id from nccl_unique_id() on rank 0"""
        b = C.create_string_buffer(bytes(uid), len(uid))
        check(lib().pb_state_shard(self.h, int(rank), int(world), b))

    def kernels_per_token(self):
        r = lib().pb_decode_kernels_per_token(self.h)
        if r < 0:
            raise PBError(r, last_error())
        return r

    def time_step_kernel(self, which, iters, stream=None):
        ms, nb = C.c_float(), C.c_double()
        check(lib().pb_time_step_kernel(self.model.h, self.h, which, iters, C.byref(ms), C.byref(nb),
                                        _stream(stream)))
        return ms.value, nb.value

    def debug_ptr(self, which):
        p = C.c_void_p()
        n = C.c_size_t()
        check(lib().pb_state_debug(self.h, which, C.byref(p), C.byref(n)))
        return p.value, n.value

    def debug_tensor(self, which, dtype):
        """copy of an internal buffer (0 kv, 1 rings, 2 final residual, 3 logits)."""
        import torch
        p, n = self.debug_ptr(which)
        esz = torch.tensor([], dtype=dtype).element_size()
        out = torch.empty(n // esz, dtype=dtype, device="cuda")
        torch.cuda.synchronize()
        out.view(torch.uint8).copy_(_view_device(p, n))
        return out

    def destroy(self):
        if self.h:
            lib().pb_state_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


def _view_device(ptr, nbytes):
    """A torch uint8 view of raw device memory owned by the library."""
    import torch

    class _A:
        pass
    a = _A()
    a.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                  "version": 3, "strides": None}
    return torch.as_tensor(a, device="cuda")


class Bonsai:
    """The Bonsai Q1_0 decoder (fwd8.c token step) on one GPU. `cfg` holds
    hidden, inter, n_layers, n_heads, n_kv, vocab, rope_factor, rope_orig_ctx,
    rope_base, attn_scale; `weights` is shaped like
    pulsar_b200.synth.make_bonsai_weights (Q1_0 18-byte blocks per tensor)."""

    SLOTS = {"q": 0, "k": 1, "v": 2, "o": 3, "gate": 4, "up": 5, "down": 6}
    NORMS = {"attn_norm": 0, "ffn_norm": 1, "q_norm": 2, "k_norm": 3}

    def __init__(self, cfg, weights=None, device=0, stream=None):
        import numpy as np
        c = BonsaiCfg(cfg["hidden"], cfg["inter"], cfg["n_layers"], cfg["n_heads"], cfg["n_kv"],
                      cfg["vocab"], cfg["rope_factor"], cfg["rope_orig_ctx"], cfg["rope_base"],
                      cfg["attn_scale"])
        h = C.c_void_p()
        check(lib().pb_bonsai_create(C.byref(c), device, C.byref(h)))
        self.h, self.cfg = h, dict(cfg)
        if weights is not None:
            st = _stream(stream)
            for li, lw in enumerate(weights["layers"]):
                for name, slot in self.SLOTS.items():
                    self.set_q1(li, slot, lw[name], st)
                for name, slot in self.NORMS.items():
                    self.set_norm(li, slot, lw[name], st)
            self.set_q1(-1, 16, weights["embed"], st)
            if weights.get("head") is not None:
                self.set_q1(-1, 17, weights["head"], st)
            self.set_norm(-1, 16, weights["out_norm"], st)

    def set_q1(self, layer, slot, blocks, st=None):
        """blocks: Q1_0 bytes [rows][K/128][18], numpy (host) or a CUDA tensor"""
        import numpy as np
        st = st if st is not None else _stream()
        if hasattr(blocks, "is_cuda") and blocks.is_cuda:
            _produced(blocks)
            check(lib().pb_bonsai_set_q1(self.h, layer, slot, C.c_void_p(blocks.data_ptr()), 1, st))
            return
        b = np.ascontiguousarray(blocks, dtype=np.uint8)
        check(lib().pb_bonsai_set_q1(self.h, layer, slot, b.ctypes.data_as(C.c_void_p), 0, st))

    def set_norm(self, layer, slot, w, st=None):
        import numpy as np
        a = np.ascontiguousarray(w, dtype=np.float32)
        check(lib().pb_bonsai_set_norm(self.h, layer, slot, a.ctypes.data_as(C.c_void_p), 0,
                                       st if st is not None else _stream()))

    def new_state(self, max_ctx, kv_bits=0):
        return BonsaiState(self, max_ctx, kv_bits)

    def close(self):
        if self.h:
            lib().pb_bonsai_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class BonsaiState:
    """One sequence: K/V cache (f16, or TurboQuant-coded when kv_bits is 3, 4
    or 43) and rope table (pb_bonsai_state)."""

    def __init__(self, model, max_ctx, kv_bits=0):
        h = C.c_void_p()
        if kv_bits:
            check(lib().pb_bonsai_state_create_tq(model.h, max_ctx, int(kv_bits), C.byref(h)))
        else:
            check(lib().pb_bonsai_state_create(model.h, max_ctx, C.byref(h)))
        self.h, self.model, self.max_ctx, self.kv_bits = h, model, max_ctx, kv_bits

    def decode(self, token, pos, x=None, logits=None, want_id=True, stream=None):
        """one token; returns the greedy id (synchronises) when want_id."""
        out = C.c_int(-1)
        check(lib().pb_bonsai_decode(self.model.h, self.h, int(token), int(pos), _ptr(x), _ptr(logits),
                                     C.byref(out) if want_id else None, _stream(stream)))
        return out.value if want_id else None

    def decode_greedy(self, token, pos, n, ids, stream=None):
        check(lib().pb_bonsai_decode_greedy(self.model.h, self.h, int(token), int(pos), int(n), _ptr(ids),
                                            _stream(stream)))

    def kv(self, layer, which):
        """torch int16 view [n_kv][max_ctx][128] of a layer's K (0) or V (1) cache"""
        import torch
        p = C.c_void_p()
        check(lib().pb_bonsai_state_kv(self.h, layer, which, C.byref(p)))
        c = self.model.cfg
        n = c["n_kv"] * self.max_ctx * 128 * 2
        return _view_device(p.value, n).view(torch.int16).view(c["n_kv"], self.max_ctx, 128)

    def residual(self, out, stream=None):
        check(lib().pb_bonsai_state_residual(self.h, _ptr(out), _stream(stream)))

    def status(self, stream=None):
        check(lib().pb_bonsai_state_status(self.h, _stream(stream)))

    def fallbacks(self):
        v = C.c_int(0)
        check(lib().pb_bonsai_state_fallbacks(self.h, C.byref(v)))
        return v.value

    def destroy(self):
        if self.h:
            lib().pb_bonsai_state_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass

