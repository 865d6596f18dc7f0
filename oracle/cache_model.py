"""Host-side model of the hot-expert cache policy.

TEST INFRASTRUCTURE ONLY (the parity checker for the product's registry and
promotion step). Restates kernels/moe-cache.cu of the reference project:

  slot sizing ........ moe_get_or_create          moe-cache.cu:542-561
  seeding ............ moe_get_or_create          moe-cache.cu:584-609
  kernel bookkeeping . moe_cache_gemv             moe-cache.cu:156-177, 180-198
                       (every (pick, token) stamps stamps[e] = clock and logs
                       a miss for a host-tagged entry, else counts a hit)
  promotion step ..... ggml_cuda_moe_cache_step   moe-cache.cu:669-775
  victim choice ...... moe_acquire_slot           moe-cache.cu:628-667

One deliberate difference: the reference appends misses to its log in
atomicAdd order, so the entries of one launch arrive in block-scheduling order
and the resulting cache state can vary run to run. The product and this model
process one step's misses sorted by (tensor id << 12 | expert). Tensor ids grow
in registration order, which is launch order for a fixed graph, so the sorted
order is one of the orders the reference can itself produce.
"""

MAX_PROMOTIONS = 48        # moe-cache.cu:37
ADMISSION_GC = 8192        # moe-cache.cu:766
SAFETY_MARGIN = 2 << 30    # moe-cache.cu:553


class TensorState:
    def __init__(self, tid, name, n_experts, expert_bytes, n_slots):
        self.id = tid
        self.name = name
        self.n_experts = n_experts
        self.expert_bytes = expert_bytes
        self.n_slots = n_slots
        self.slot_of = [-1] * n_experts
        self.expert_of = [-1] * n_slots
        self.stamps = [0] * n_experts


class CacheModel:
    def __init__(self, slots=320, budget_bytes=30 << 30, seed=None, free_vram=1 << 62):
        self.slots_cfg = max(0, slots)
        self.budget = budget_bytes
        self.used = 0
        self.free_vram = free_vram
        self.seed = seed or {}
        self.tensors = []
        self.by_key = {}
        self.clock = 0
        self.admission = {}
        self.log = []
        self.hits = 0
        self.promotions = 0

    # -- registration (moe-cache.cu:525-622) --------------------------------
    def register(self, key, name, n_experts, expert_bytes):
        if key in self.by_key:
            return self.by_key[key]
        slots = self.slots_cfg
        free_budget = self.budget - self.used if self.budget > self.used else 0
        if slots * expert_bytes > free_budget:
            slots = free_budget // expert_bytes
        usable = self.free_vram - SAFETY_MARGIN if self.free_vram > SAFETY_MARGIN else 0
        if slots * expert_bytes > usable:
            slots = usable // expert_bytes
        slots = min(slots, n_experts)
        t = TensorState(len(self.tensors), name, n_experts, expert_bytes, slots)
        self.used += slots * expert_bytes
        self.tensors.append(t)
        self.by_key[key] = t
        if name in self.seed and slots > 0:
            seeded = 0
            for e in self.seed[name]:
                if seeded >= slots:
                    break
                if e < 0 or e >= n_experts or t.slot_of[e] >= 0:
                    continue
                t.slot_of[e] = seeded
                t.expert_of[seeded] = e
                seeded += 1
        return t

    # -- one kernel launch's bookkeeping ------------------------------------
    def launch(self, t, experts):
        """experts: expert id of every (pick, token) entry of one launch."""
        for e in experts:
            t.stamps[e] = self.clock
            if t.slot_of[e] < 0:
                self.log.append((t.id << 12) | e)
            else:
                self.hits += 1

    # -- victim selection (moe-cache.cu:628-667) ----------------------------
    def _acquire_slot(self, t):
        if t.n_slots == 0:
            return -1
        for s in range(t.n_slots):
            if t.expert_of[s] < 0:
                return s
        victim_slot, best = -1, 0xFFFFFFFF
        for s in range(t.n_slots):
            e = t.expert_of[s]
            stamp = t.stamps[e] if e >= 0 else 0
            if stamp < best:
                best, victim_slot = stamp, s
        if victim_slot < 0:
            return -1
        victim = t.expert_of[victim_slot]
        if victim >= 0:
            t.slot_of[victim] = -1
        t.expert_of[victim_slot] = -1
        return victim_slot

    # -- promotion step (moe-cache.cu:669-775) ------------------------------
    def step(self):
        log = sorted(self.log)
        self.log = []
        self.clock += 1
        promoted = 0
        for packed in log:
            if promoted >= MAX_PROMOTIONS:
                break
            cnt = self.admission.get(packed, 0) + 1
            self.admission[packed] = cnt
            if cnt < 2:
                continue
            self.admission[packed] = 0
            cid, e = packed >> 12, packed & 0xFFF
            if cid < 0 or cid >= len(self.tensors):
                continue
            t = self.tensors[cid]
            if e < 0 or e >= t.n_experts or t.slot_of[e] >= 0:
                continue
            slot = self._acquire_slot(t)
            if slot < 0:
                continue
            t.slot_of[e] = slot
            t.expert_of[slot] = e
            promoted += 1
            self.promotions += 1
        if len(self.admission) > ADMISSION_GC:
            self.admission = {k: v for k, v in self.admission.items() if v != 0}
        return promoted


def parse_seed(text):
    """Seed-file format of moe-cache.cu:483-523: 'tensorname id,id,...' per line."""
    seed = {}
    for line in text.splitlines():
        if " " not in line:
            continue
        name, rest = line.split(" ", 1)
        ids = []
        for tok in rest.strip().split(","):
            tok = tok.strip()
            if not tok:
                break
            try:
                ids.append(int(tok))
            except ValueError:
                break
        seed[name] = ids
    return seed
