"""SSD (Subnetwork Speculative Decoding) round on B200: drop-in for the
reference's ssd.engine / ssd.models API, computed by the sm_100a kernels in
libssd_b200.so (see include/ssd_b200.h)."""

__version__ = "0.1.0"
