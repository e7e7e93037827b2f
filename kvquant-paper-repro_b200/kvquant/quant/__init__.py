from .nuq import train_nuq_codebook
from .dense_sparse import extract_outliers, pack_csr, unpack_csr
from .kv_quantizer import KVQuantizer

__all__ = [
    "train_nuq_codebook",
    "extract_outliers",
    "pack_csr",
    "unpack_csr",
    "KVQuantizer",
]
