---------------------------- MODULE BroadcastChainN ----------------------------
(* One block index of the Broadcast push chain: ranks 0 -> 1 -> ... -> N-1 *)
(* (rank 0 the root), S steps. The root stores piece k into rank 1's output *)
(* and publishes flag[1] = k + 1. Rank r in 1..N-2 waits until flag[r] >=   *)
(* k + 1 (unless SkipWait), reads piece k from its own output, stores it     *)
(* into rank r+1's output and publishes flag[r+1] = k + 1.                   *)
EXTENDS Integers

CONSTANTS N, S, SkipWait
VARIABLES k, ph, flag, got, bad
vars == <<k, ph, flag, got, bad>>

Ranks == 0..(N - 1)
Senders == 0..(N - 2)
Steps == 0..(S - 1)

Init == /\ k = [r \in Ranks |-> 0] /\ ph = [r \in Ranks |-> 0]
        /\ flag = [r \in Ranks |-> 0]
        /\ got = [r \in Ranks |-> IF r = 0 THEN Steps ELSE {}]
        /\ bad = FALSE

Wait(r) == /\ k[r] < S /\ ph[r] = 0
           /\ r = 0 \/ SkipWait \/ flag[r] >= k[r] + 1
           /\ ph' = [ph EXCEPT ![r] = 1]
           /\ UNCHANGED <<k, flag, got, bad>>

Read(r) == /\ k[r] < S /\ ph[r] = 1
           /\ bad' = (bad \/ k[r] \notin got[r])
           /\ ph' = [ph EXCEPT ![r] = 2]
           /\ UNCHANGED <<k, flag, got>>

Write(r) == /\ k[r] < S /\ ph[r] = 2
            /\ got' = [got EXCEPT ![r + 1] = IF k[r] \in got[r] THEN got[r + 1] \cup {k[r]}
                                             ELSE got[r + 1]]
            /\ flag' = [flag EXCEPT ![r + 1] = k[r] + 1]
            /\ k' = [k EXCEPT ![r] = k[r] + 1] /\ ph' = [ph EXCEPT ![r] = 0]
            /\ UNCHANGED bad

Done == \A r \in Senders : k[r] = S

Next == \/ \E r \in Senders : Wait(r) \/ Read(r) \/ Write(r)
        \/ (Done /\ UNCHANGED vars)

Spec == Init /\ [][Next]_vars

ForwardedArrived == ~bad
AllPiecesDelivered == Done => \A r \in Ranks : got[r] = Steps
=============================================================================
