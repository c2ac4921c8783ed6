"""Writes GGUF files for the loader tests with the third-party `gguf` 0.19.0 package."""
import numpy as np


def write_gguf(path, tensors, arch="flux"):
    """tensors: {name: QTensorRef-like (ggml_type, shape, raw)} in the oracle's layout
    (matrices [rows, cols] of raw GGML bytes; 1-D F32 vectors)."""
    import gguf
    w = gguf.GGUFWriter(str(path), arch)
    for name, qt in tensors.items():
        t, shape, raw = qt.ggml_type, tuple(qt.shape), np.asarray(qt.raw, dtype=np.uint8)
        if t == 0:
            w.add_tensor(name, raw.view(np.float32).reshape(shape))
        else:
            rows = int(np.prod(shape[:-1])) if len(shape) > 1 else 1
            w.add_tensor(name, raw.reshape(rows, -1), raw_dtype=gguf.GGMLQuantizationType(t))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
