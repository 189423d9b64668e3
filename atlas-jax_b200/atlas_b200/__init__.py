"""B200-native Atlas chunked deep-memory scan (host side of libatlas_scan.so)."""
from ._lib import (ATLAS_BF16, ATLAS_F32, ATLAS_PREC_EXACT, ATLAS_PREC_TENSOR, ATLAS_PREC_TENSOR_BATCHED, AtlasError,  # noqa: F401
                   AtlasScanParams, load)
from .scan import (AtlasScan, ScanConfig, atlas_scan, device_status, linear_scan_backward, linear_scan_forward,  # noqa: F401,E501
                   polar_express, scan_backward, scan_forward)
