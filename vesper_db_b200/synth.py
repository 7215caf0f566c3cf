"""Seeded synthetic data of the benchmark workloads, generated on the device.

IVF-PQ search: a mixture of `n_centres` anisotropic Gaussians in `dim` dimensions:
centres ~U[-1, 1], per-centre per-dimension sigma ~U[0.01, 0.2]; rows pick a centre
uniformly.  Base rows come in fixed-size chunks (chunk c drawn with seed 1234 + c) so
any subset of chunks can be generated independently -- on one GPU or sharded across
ranks.  Queries use seed 5678.  k-means training and the sharded search use isotropic
mixtures (`gen_isotropic_mixture`).  Used by bench.py.
"""
from __future__ import annotations

CENTRE_SEED = 42
BASE_SEED = 1234
QUERY_SEED = 5678


def gen_centres(torch, dev, n_centres: int, dim: int):
    g = torch.Generator(device=dev)
    g.manual_seed(CENTRE_SEED)
    centres = torch.rand(n_centres, dim, generator=g, device=dev) * 2 - 1
    sigmas = torch.rand(n_centres, dim, generator=g, device=dev) * 0.19 + 0.01
    return centres, sigmas


def gen_rows(torch, dev, centres, sigmas, n: int, seed: int, out=None):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    lab = torch.randint(0, centres.shape[0], (n,), generator=g, device=dev)
    noise = torch.randn(n, centres.shape[1], generator=g, device=dev)
    x = centres[lab].addcmul_(sigmas[lab], noise)
    if out is not None:
        out.copy_(x)
        return out
    return x


def gen_base_chunk(torch, dev, centres, sigmas, c: int, chunk: int, out=None):
    return gen_rows(torch, dev, centres, sigmas, chunk, BASE_SEED + c, out)


def gen_queries(torch, dev, centres, sigmas, nq: int):
    return gen_rows(torch, dev, centres, sigmas, nq, QUERY_SEED)


def gen_isotropic_mixture(torch, dev, n_centres: int, dim: int, sigma: float, n: int, seed: int, out=None):
    """n rows from a mixture of n_centres isotropic Gaussians (centres ~U[-1, 1], drawn
    with seed CENTRE_SEED; every row picks a centre uniformly; noise sigma), seeded by
    `seed`.  The k-means training workload: 2,000,000 x 128 rows of 20,000 centres,
    sigma 0.05."""
    g = torch.Generator(device=dev)
    g.manual_seed(CENTRE_SEED)
    centres = torch.rand(n_centres, dim, generator=g, device=dev) * 2 - 1
    g.manual_seed(seed)
    lab = torch.randint(0, n_centres, (n,), generator=g, device=dev)
    x = centres[lab].add_(torch.randn(n, dim, generator=g, device=dev), alpha=sigma)
    if out is not None:
        out.copy_(x)
        return out
    return x
