"""LAN pairing: BLAKE3 against published test vectors, the commitment and SAS against the
frozen pairing vectors of the protocol, and the commit / challenge / reveal state machines."""
import pytest

from syntropy_b200.cluster.pairing import (Joiner, Keyholder, PairingError, Sas, blake3, commitment, opens, sas,
                                           sas_digest)

# BLAKE3 of inputs whose byte i is i % 251 (the published test-vector input), by length:
# one block, one chunk, chunk + 1 byte (a parent node), two chunks
BLAKE3_VECTORS = {
    0: "af1349b9f5f9a1a6a0404dea36dcc9499bcb25c9adc112b7cc9a93cae41f3262",
    1: "2d3adedff11b61f14c886e35afa036736dcd87a74d27b5c1510225d0f592e213",
    1023: "10108970eeda3eb932baac1428c7a2163b0e924c9a9e25b35bba72b28f70bd11",
    1024: "42214739f095a406f3fc83deb889744ac00df831c10daa55189b5d121c855af7",
    1025: "d00278ae47eb27b34faecf67b4fe263f82d5412916c1ffd97c8cb7fb814b8444",
    2048: "e776b6028c7cd22a4d0ba182a8bf62205d2ef576467e838ed6f2529b85fba24a",
}


def _seq(a, n):
    return bytes(range(a, a + n))


def _h(s):
    return bytes.fromhex(s)


# (cluster_id, joiner, keyholder, nonce_c, nonce_k, commit, sas digest, sas, shown)
COUNT = (_seq(0, 32), _seq(32, 32), _seq(64, 32), _seq(96, 16), _seq(112, 16))
PAIRING_VECTORS = [
    ((bytes(32), bytes(32), bytes(32), bytes(16), bytes(16)),
     "0525d617e1502da455a48016817d1d5cba22fb9544d18c4c63d43c7aea3a7ff8",
     "9f8961aa6530a88d5e8205906ad413324b7ca6adfb5c63e2dc13c68e936c173c", 518943, "518 943"),
    (COUNT, "7aeaa0b67490f57778f63e6925b8095fe30477415e85da34a635232e35d8e0e3",
     "91d59c0e807e764082c3346b049902c1e6a6ef4b46110dabcb063f000f4fcf79", 159313, "159 313"),
    ((COUNT[0], COUNT[2], COUNT[1], COUNT[3], COUNT[4]),  # roles swapped: another code
     "3ffc6b5da48e064cf69db42d7e9948fd89ef513f687059a43672cd5d608087ba",
     "adaafeb46457cc40dc4b5b73112a0c5e1cab6a95e6901eba5a0efcec8a9fc51d", 588717, "588 717"),
    ((_h("55ff00770784c8db495049afdf645e21316c6b5338c3e89ee21133cc2b98ff70"),
      _h("a8b23a4f469b01f698f4f4700adc53ab71833ded3aabb52cdec6d5f0b3f17c9a"),
      _h("1949701bcd2d0d3e98e530927990fd2772d960ed8d500920dd578fc3b83a9617"),
      _h("c5fa7a4403a7d75451fa0c8627fccdb0"), _h("cc459b73d08c9671b27a6bae4ba228f1")),
     "50d734198615aa5356ceb6551c98d30141e1df752ae762a06666435d48a1e8bf",
     "aa07a592f2089b21b4324c0271691e1002dbda9a4a2a5dfba51a4e6cb3d730f3", 288938, "288 938"),
    ((COUNT[0], COUNT[1], COUNT[2], COUNT[3], _h("707172737475767778797a7b7c7d024e")),  # leading zeros
     "7aeaa0b67490f57778f63e6925b8095fe30477415e85da34a635232e35d8e0e3",
     "4e58200e3a66a5c87336481e98a337f10f1f18af47dee200b6f589e2f9b7ec6d", 782, "000 782"),
]


@pytest.mark.parametrize("n", sorted(BLAKE3_VECTORS))
def test_blake3_vectors(n):
    assert blake3(bytes(i % 251 for i in range(n))).hex() == BLAKE3_VECTORS[n]


def test_blake3_many_chunks_is_a_tree():
    # 5 chunks: the last chunk is merged with a 4-chunk left subtree; lengths around chunk edges differ
    digests = {blake3(bytes(i % 251 for i in range(n))) for n in (4095, 4096, 4097, 5120, 5121, 8193)}
    assert len(digests) == 6 and all(len(d) == 32 for d in digests)


@pytest.mark.parametrize("vec", PAIRING_VECTORS, ids=["zeros", "counting", "roles-swapped", "seeded", "leading-zeros"])
def test_pairing_vectors(vec):
    (cid, joiner, keyholder, nc, nk), commit, digest, code, shown = vec
    assert commitment(joiner, nc).hex() == commit
    assert opens(_h(commit), joiner, nc)
    assert sas_digest(cid, joiner, keyholder, nc, nk).hex() == digest
    s = sas(cid, joiner, keyholder, nc, nk)
    assert s == Sas(code) and str(s) == shown


def test_exchange_and_rejections():
    cid, jid, kid = _seq(0, 32), _seq(32, 32), _seq(64, 32)
    j, k = Joiner(cid, jid, kid), Keyholder(cid, kid, jid)
    with pytest.raises(PairingError):
        j.on_challenge(bytes(16))          # no reveal before our own commitment
    commit = j.request()
    nonce_k = k.on_request(commit)
    with pytest.raises(PairingError):
        k.code()                           # no code before the reveal
    k.on_reveal(j.on_challenge(nonce_k))
    assert j.code() == k.code()
    # a reveal that does not open the commitment is denied
    j2, k2 = Joiner(cid, jid, kid), Keyholder(cid, kid, jid)
    nk2 = k2.on_request(j2.request())
    j2.on_challenge(nk2)
    with pytest.raises(PairingError, match="denied"):
        k2.on_reveal(bytes(16))
    # a relay that swaps in its own nonce makes the codes differ
    j3, k3 = Joiner(cid, jid, kid, nonce_c=_seq(96, 16)), Keyholder(cid, kid, jid, nonce_k=_seq(112, 16))
    k3.on_request(j3.request())
    j3.on_challenge(bytes(16))             # the attacker's nonce, not the keyholder's
    k3.on_reveal(j3.nonce_c)
    assert j3.code() != k3.code()
    with pytest.raises(ValueError):
        commitment(jid[:31], bytes(16))
