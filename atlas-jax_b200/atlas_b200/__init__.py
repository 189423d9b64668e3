"""B200-native Atlas chunked deep-memory scan (host side of libatlas_scan.so)."""
from ._lib import (ATLAS_BF16, ATLAS_F32, ATLAS_PREC_EXACT, ATLAS_PREC_TENSOR, AtlasError,  # noqa: F401
                   AtlasScanParams, load)
from .scan import (AtlasScan, ScanConfig, atlas_scan, device_status, polar_express,  # noqa: F401
                   scan_backward, scan_forward)
