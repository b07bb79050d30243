"""When the peer-memory kernels may serve a group: every rank on this host,
on a distinct GPU that this process sees and can address. Checked on the
decision function with made-up hosts, PCI ids and peer-access answers."""

from dstraining_b200.parallel.topology import SINGLE, peer_reachable, peers_addressable

HOST_A, HOST_B = "node-a/boot-1", "node-b/boot-2"
VISIBLE = {f"0000:{b:02x}:00": i for i, b in enumerate((0x18, 0x2a, 0x3a, 0x5d))}


def _all(a, b):
    return True


def test_one_host_all_visible():
    infos = [(HOST_A, "0000:18:00"), (HOST_A, "0000:2a:00"), (HOST_A, "0000:3a:00")]
    assert all(peers_addressable(infos, r, VISIBLE, _all) for r in range(3))


def test_group_across_machines():
    infos = [(HOST_A, "0000:18:00"), (HOST_B, "0000:18:00")]
    assert not peers_addressable(infos, 0, VISIBLE, _all)
    assert not peers_addressable(infos, 1, VISIBLE, _all)


def test_same_host_name_other_machine():
    infos = [("node/boot-1", "0000:18:00"), ("node/boot-2", "0000:2a:00")]
    assert not peers_addressable(infos, 0, VISIBLE, _all)


def test_peer_gpu_not_visible_or_not_addressable():
    infos = [(HOST_A, "0000:18:00"), (HOST_A, "0000:99:00")]
    assert not peers_addressable(infos, 0, VISIBLE, _all)  # peer's GPU hidden from this process
    infos = [(HOST_A, "0000:18:00"), (HOST_A, "0000:2a:00")]
    assert not peers_addressable(infos, 0, VISIBLE, lambda a, b: False)  # no P2P path
    assert peers_addressable(infos, 0, VISIBLE, lambda a, b: {a, b} == {0, 1})


def test_two_ranks_one_gpu():
    infos = [(HOST_A, "0000:18:00"), (HOST_A, "0000:18:00")]
    assert not peers_addressable(infos, 0, VISIBLE, _all)


def test_single_rank_and_cpu():
    assert peer_reachable(SINGLE)
