"""Attention beyond the dense GQA decode kernel: MLA over an NVFP4 latent cache and DSA-style sparse selection."""
