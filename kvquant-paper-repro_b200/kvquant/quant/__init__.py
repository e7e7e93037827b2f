from .nuq import fit_nuq_codebook_cuda, train_nuq_codebook
from .dense_sparse import extract_outliers, pack_csr, unpack_csr
from .kv_quantizer import KVQuantizer

__all__ = [
    "train_nuq_codebook",
    "fit_nuq_codebook_cuda",
    "extract_outliers",
    "pack_csr",
    "unpack_csr",
    "KVQuantizer",
]
