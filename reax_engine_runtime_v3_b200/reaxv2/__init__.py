"""Drop-in replacements for the reference's ``reaxv2`` gate/up modules (B200 kernels behind them)."""
