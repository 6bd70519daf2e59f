"""Synthetic GGUF files for the format tests, written with gguf-py (the
writer the reference's converter uses, scripts/objects/gguf_schema.py), and
gguf-py's numpy dequantisers as the independent statement of GGML's block
formats."""
import numpy as np
import gguf
from gguf import GGMLQuantizationType as Q
from gguf import quants

QTYPES = {"f32": Q.F32, "f16": Q.F16, "bf16": Q.BF16, "q8_0": Q.Q8_0, "q4_0": Q.Q4_0, "q4_1": Q.Q4_1,
          "q4_k": Q.Q4_K}


def random_q4_k(rows: int, cols: int, seed: int) -> np.ndarray:
    """Random Q4_K blocks [rows, cols / 256 * 144] (gguf-py cannot quantise
    to Q4_K): finite f16 d / dmin, random scale and quant bytes."""
    rng = np.random.default_rng(seed)
    nb = rows * cols // 256
    blk = rng.integers(0, 256, size=(nb, 144), dtype=np.uint8)
    blk[:, 0:2] = np.frombuffer(rng.uniform(0.001, 0.05, nb).astype(np.float16).tobytes(), np.uint8).reshape(nb, 2)
    blk[:, 2:4] = np.frombuffer(rng.uniform(0.0, 0.05, nb).astype(np.float16).tobytes(), np.uint8).reshape(nb, 2)
    return blk.reshape(rows, -1)


def stored(x: np.ndarray, dtype: str, seed: int = 0):
    """(array to write, raw_dtype or None) for a float32 matrix in `dtype`."""
    if dtype == "f32":
        return x.astype(np.float32), None
    if dtype == "f16":
        return x.astype(np.float16), None
    if dtype == "bf16":
        return quants.quantize(x, Q.BF16), Q.BF16
    if dtype == "q4_k":
        return random_q4_k(x.shape[0], x.shape[1], seed), Q.Q4_K
    return quants.quantize(x, QTYPES[dtype]), QTYPES[dtype]


def dequantized(arr: np.ndarray, raw_dtype) -> np.ndarray:
    """float32 values of what `stored` wrote (gguf-py dequantisation)."""
    if raw_dtype is None:
        return arr.astype(np.float32)
    return quants.dequantize(arr, raw_dtype).astype(np.float32)


def write(path: str, tensors: dict, kv: dict | None = None, arch: str = "sam3d.test"):
    """tensors: name -> float32 array or (stored array, raw_dtype); kv: key ->
    python value (int -> u32, float -> f32, str, list of int / str)."""
    w = gguf.GGUFWriter(path, arch)
    for k, v in (kv or {}).items():
        if isinstance(v, bool):
            w.add_bool(k, v)
        elif isinstance(v, int):
            w.add_uint32(k, v)
        elif isinstance(v, float):
            w.add_float32(k, v)
        elif isinstance(v, str):
            w.add_string(k, v)
        else:
            w.add_array(k, v)
    for name, t in tensors.items():
        if isinstance(t, tuple):
            arr, raw = t
            if raw is None:
                w.add_tensor(name, arr)
            else:
                w.add_tensor(name, arr, raw_shape=arr.shape, raw_dtype=raw)
        else:
            w.add_tensor(name, t)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
