"""SHA-256 pins of the frozen ICTC harmonic basis, version v1.

Each digest is taken over the row-major float64 bytes of the (Dsym(l), 2l+1)
basis matrix for degree l.  The values are the ones the ICTC-O3 reference pins
(``ictc_o3/basis/ictd_irreps.py:633-647``); they have to be identical because
the basis is a data format shared with released checkpoints.
"""

BASIS_VERSION = "v1"

BASIS_SHA256 = {
    0: "6c3c396ed6b5c36dcae172271f462051b1266b851e92df3deea8ac65478fd712",
    1: "1332df685c45a61a0ac008a6a653295b8c5655361c1d34b6304b22ec40235fb8",
    2: "0881fbfd2a1866b76334d823d216ec74773a91a5f77234c45bb956838df7c315",
    3: "a7440553d51231cc044287b305d35cb5cafc59f77d7528d8189956c51a52a9e0",
    4: "f89f4b7f49ed9be8cc7fbbcec5e1a8947442c612d239bd42ce36180c6c644225",
    5: "8cce9bfb0a710f2c19d50ca3bcf6a79593697b5bd129085f10422066c2030ea8",
    6: "01cc08fe54c00daaff6899a86c923b62433f1691b7f283b95643c7be78ce9a96",
}
