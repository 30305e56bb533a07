"""Parameters of the binning stress fixtures, shared by the generator and the tests."""
STRESS_CASES = [
    # (name, seed, G, H, W, R, K, stress_mu2d keyword arguments)
    ("tiny_k8", 11, 400, 48, 64, 1, 8, dict(n_clusters=4, sigma_px=5.0)),
    ("ties_k32", 12, 3000, 64, 64, 1, 32, dict(n_clusters=6, sigma_px=4.0, quantise=True)),
    ("special_k16", 13, 2000, 64, 96, 1, 16, dict(n_clusters=5, sigma_px=8.0, n_special=24)),
    ("r2_k64", 14, 5000, 96, 128, 2, 64, dict(n_clusters=10, sigma_px=6.0)),
    ("sparse_k128", 15, 300, 256, 256, 1, 128, dict(n_clusters=30, sigma_px=20.0, frac_off=0.3)),
    ("allout_k4", 16, 200, 32, 32, 1, 4, dict(n_clusters=2, sigma_px=3.0, frac_drop=1.0)),
]

# the largest stencil radius the entry points accept (R = 3: a 7x7 tile neighbourhood per cell)
RADIUS_CASES = [
    ("r3_k48", 17, 4000, 80, 112, 3, 48, dict(n_clusters=8, sigma_px=7.0)),
    ("r3_k8_ties", 18, 1500, 64, 64, 3, 8, dict(n_clusters=3, sigma_px=4.0, quantise=True)),
    ("r3_k128_sparse", 19, 500, 256, 320, 3, 128, dict(n_clusters=3, sigma_px=6.0, frac_off=0.3)),
]

BIG_CASE = dict(seed=31, G=1_000_000, H=1072, W=1920, R=1, K=256,
                kw=dict(n_clusters=64, sigma_px=30.0, frac_off=0.05, frac_drop=0.02))
