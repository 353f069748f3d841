"""flashinfer-bench solution packaging for the B200 GDN kernels."""
