"""Z4-linear Kerdock / Delsarte-Goethals codebooks for the switch checkpoint format.

The reference's coded-memory switch stores a ``[capacity, N]`` fp32 codebook
(``model.switch.codebook``) of unit vectors with low mutual coherence, built
from the Z4-linear Kerdock code K(m) (or DG(m, 1)) through the Gray map
(reference: src/granite_switch/hf/switch/codes/code_generator.py:20-236). The
buffer is part of the checkpoint, so the composer here writes one and the
loader reads it back. This runtime routes with the exact scan in
:mod:`.scan`, so the codebook is only needed for format parity and for the
coded-memory oracle in :mod:`.coded_switch`.

Construction (Hammons, Kumar, Calderbank, Sloane and Sole, "The Z4-linearity of
Kerdock, Preparata, Goethals and related codes", IEEE Trans. IT 1994):

* r = m - 1 (odd). Lift a primitive binary polynomial of degree r to its basic
  primitive polynomial h over Z4 with Graeffe's root-squaring step
  h(x^2) = +-(e(x)^2 - o(x)^2), where e/o are the even/odd parts.
* xi = x mod h generates the Teichmuller set T = {0} u {xi^k : 0 <= k < 2^r - 1}.
* Tr: GR(4, r) -> Z4, Tr(a) = sum_i sigma^i(a) with Frobenius sigma(xi) = xi^2.
* Kerdock codeword for (lambda, eps): c(x) = Tr(lambda x) + eps over x in T,
  lambda in GR(4, r), eps in Z4. DG(m, 1) adds 2 Tr(mu x^3), mu in T.
* Gray map 0->00, 1->01, 2->11, 3->10 gives binary length 2^m; the vector is
  (-1)^bits / sqrt(2^m). eps and eps + 2 give antipodal vectors, so one of each
  pair (eps in {0, 1}) is kept: Kerdock capacity 2^(2m-1), coherence 2^(-m/2).
"""
from __future__ import annotations

import itertools

import numpy as np
import torch

# Primitive binary polynomials, coefficients low -> high degree.
_PRIMITIVE = {
    3: [1, 1, 0, 1],            # 1 + x + x^3
    5: [1, 0, 1, 0, 0, 1],      # 1 + x^2 + x^5
    7: [1, 1, 0, 0, 0, 0, 0, 1],  # 1 + x + x^7
    9: [1, 0, 0, 0, 1, 0, 0, 0, 0, 1],  # 1 + x^4 + x^9
}


def _polymul(a, b, mod=4):
    out = [0] * (len(a) + len(b) - 1)
    for i, x in enumerate(a):
        if x:
            for j, y in enumerate(b):
                out[i + j] = (out[i + j] + x * y) % mod
    return out


def hensel_lift(binary_poly: list[int]) -> list[int]:
    """Basic primitive polynomial over Z4 (monic) lifting a primitive binary one."""
    r = len(binary_poly) - 1
    e = [c if i % 2 == 0 else 0 for i, c in enumerate(binary_poly)]
    o = [c if i % 2 == 1 else 0 for i, c in enumerate(binary_poly)]
    sq = [(x - y) % 4 for x, y in itertools.zip_longest(_polymul(e, e), _polymul(o, o), fillvalue=0)]
    h = [sq[2 * i] for i in range(r + 1)]  # h(x^2) = e^2 - o^2  (odd terms vanish)
    if h[r] % 4 == 3:  # make monic: multiply by -1
        h = [(-c) % 4 for c in h]
    assert h[r] == 1, "lift is not monic"
    return h


class GaloisRingZ4:
    """Arithmetic in GR(4, r) = Z4[x]/(h(x)), elements as int8[r] coefficient rows."""

    def __init__(self, r: int):
        if r not in _PRIMITIVE:
            raise ValueError(f"unsupported extension degree {r}")
        self.r = r
        self.h = hensel_lift(_PRIMITIVE[r])
        self.order = 2 ** r - 1
        # powers of xi
        pw = np.zeros((self.order, r), dtype=np.int64)
        cur = np.zeros(r, dtype=np.int64)
        cur[0] = 1
        for k in range(self.order):
            pw[k] = cur
            cur = self._mul_x(cur)
        assert np.array_equal(cur, pw[0]), "xi does not have order 2^r - 1"
        self.powers = pw
        # Tr(xi^k) for every k: sum over the Frobenius orbit xi^(k 2^i)
        tr = np.zeros(self.order, dtype=np.int64)
        for k in range(self.order):
            acc = np.zeros(r, dtype=np.int64)
            for i in range(r):
                acc = (acc + pw[(k * (2 ** i)) % self.order]) % 4
            assert np.all(acc[1:] == 0), "trace is not in Z4"
            tr[k] = acc[0]
        self.trace_pow = tr

    def _mul_x(self, a: np.ndarray) -> np.ndarray:
        r = self.r
        top = a[r - 1]
        out = np.zeros(r, dtype=np.int64)
        out[1:] = a[:-1]
        # x^r = -(h_0 + ... + h_{r-1} x^{r-1})
        for i in range(r):
            out[i] = (out[i] - top * self.h[i]) % 4
        return out

    def trace_lambda_x(self, lam: np.ndarray) -> np.ndarray:
        """``Tr(lambda * x)`` for x over the Teichmuller set, in the order [0, xi^0, xi^1, ...]."""
        n = self.order + 1
        out = np.zeros(n, dtype=np.int64)
        # Tr(lam xi^t) = sum_j lam_j Tr(xi^(j + t))
        t = np.arange(self.order)
        for j in range(self.r):
            if lam[j]:
                out[1:] = (out[1:] + lam[j] * self.trace_pow[(j + t) % self.order]) % 4
        return out


_GRAY = np.array([[0, 0], [0, 1], [1, 1], [1, 0]], dtype=np.int64)


def gray_map(z4: np.ndarray) -> np.ndarray:
    """Z4 vector of length n -> binary vector of length 2n."""
    return _GRAY[z4 % 4].reshape(*z4.shape[:-1], -1)


class KerdockDGCodeGenerator:
    """Precomputes unit-norm Kerdock (``"kerdock"``) or DG(m,1) (``"dg1"``) codewords.

    ``N = 2^m`` is the vector dimension; ``capacity`` the number of codewords
    (one per antipodal pair).
    """

    def __init__(self, m: int = 6, code_type: str = "kerdock", verbose: bool = False):
        if m % 2 or m < 4:
            raise ValueError(f"m must be even and >= 4, got {m}")
        if code_type not in ("kerdock", "dg1"):
            raise ValueError(f"code_type must be 'kerdock' or 'dg1', got {code_type!r}")
        self.m = m
        self.code_type = code_type
        self.N = 2 ** m
        self.ring = GaloisRingZ4(m - 1)
        base = 2 ** (2 * m - 1)
        self.capacity = base if code_type == "kerdock" else base * 2 ** (m - 1)

    def _codeword_z4(self, index: int) -> np.ndarray:
        r = self.ring.r
        eps = index & 1
        rest = index >> 1
        lam_idx = rest % (4 ** r)
        mu_idx = rest // (4 ** r)
        lam = np.array([(lam_idx >> (2 * j)) & 3 for j in range(r)], dtype=np.int64)
        c = (self.ring.trace_lambda_x(lam) + eps) % 4
        if self.code_type == "dg1" and mu_idx > 0:
            # mu = xi^(mu_idx - 1); add 2 Tr(mu x^3) over x in T
            k = mu_idx - 1
            t = np.arange(self.ring.order)
            tr = self.ring.trace_pow[(k + 3 * t) % self.ring.order]
            c[1:] = (c[1:] + 2 * tr) % 4
        return c

    def generate_code_vectors_batch(self, indices, dtype=torch.float32) -> torch.Tensor:
        idx = list(indices)
        z4 = np.stack([self._codeword_z4(i) for i in idx])
        bits = gray_map(z4)
        vec = (1.0 - 2.0 * bits) / np.sqrt(self.N)
        return torch.tensor(vec, dtype=dtype)

    #: largest codebook written into a checkpoint (the buffer ships with every model)
    MAX_CODEBOOK_BYTES = 128 * 1024 * 1024

    def precompute_codebook(self, dtype=torch.float32) -> torch.Tensor:
        """All ``[capacity, N]`` code vectors; raises for codebooks above 128 MB (DG(8, 1):
        4.2M vectors of dimension 256), which would have to be generated on the fly."""
        size = self.capacity * self.N * 4
        if size > self.MAX_CODEBOOK_BYTES:
            raise ValueError(f"codebook of {self.capacity} x {self.N} fp32 is {size / 2**20:.0f} MB, above the "
                             f"{self.MAX_CODEBOOK_BYTES // 2**20} MB a checkpoint carries")
        return self.generate_code_vectors_batch(range(self.capacity), dtype=dtype)


def verify_coherence(codebook: torch.Tensor, sample: int | None = None) -> float:
    """Max |<c_i, c_j>| over distinct rows (optionally on the first ``sample`` rows)."""
    cb = codebook if sample is None else codebook[:sample]
    g = cb.double() @ cb.double().t()
    g.fill_diagonal_(0.0)
    return float(g.abs().max())


def recover_count_from_signal(signal: torch.Tensor, capacity: int) -> torch.Tensor:
    """Integer ``n`` from the counting head's ``1/(1+n)``; computed in fp32."""
    n = 1.0 / signal.float() - 1.0
    return torch.clamp(torch.round(n).long(), 0, capacity - 1)
