---------------------------- MODULE OneShotBarrierN ----------------------------
(* The low-latency engine's arrive/depart barriers (one block index), over *)
(* C consecutive calls on the same streams. Rank r, call c:               *)
(*  Produce: the caller's stream consumes every slice of its output of    *)
(*    call c-1 (each must hold call c-1), writes input c, and the kernel  *)
(*    arrives (arr[r] = c + 1 on every rank).                             *)
(*  Data: after every rank arrived (arr[q] >= c + 1, unless SkipArrive),  *)
(*    reads every rank's input (each must hold call c) and writes slice r *)
(*    of every rank's output (Two, the two-shot) or every slice of its    *)
(*    own output (the one-shot).                                          *)
(*  Depart: dep[r] = c + 1 on every rank.                                 *)
(*  Leave: after every rank departed (dep[q] >= c + 1, unless SkipDepart) *)
(*    the stream goes on to call c + 1.                                   *)
EXTENDS Integers

CONSTANTS N, C, Two, SkipArrive, SkipDepart
VARIABLES c, ph, arr, dep, inp, out, bad
vars == <<c, ph, arr, dep, inp, out, bad>>

Ranks == 0..(N - 1)

Init == /\ c = [r \in Ranks |-> 0] /\ ph = [r \in Ranks |-> 0]
        /\ arr = [r \in Ranks |-> 0] /\ dep = [r \in Ranks |-> 0]
        /\ inp = [r \in Ranks |-> -1]
        /\ out = [r \in Ranks |-> [s \in Ranks |-> -1]]
        /\ bad = FALSE

Produce(r) == /\ c[r] < C /\ ph[r] = 0
              /\ bad' = (bad \/ (c[r] > 0 /\ \E s \in Ranks : out[r][s] # c[r] - 1))
              /\ inp' = [inp EXCEPT ![r] = c[r]]
              /\ arr' = [arr EXCEPT ![r] = c[r] + 1]
              /\ ph' = [ph EXCEPT ![r] = 1]
              /\ UNCHANGED <<c, dep, out>>

Data(r) == /\ c[r] < C /\ ph[r] = 1
           /\ SkipArrive \/ \A q \in Ranks : arr[q] >= c[r] + 1
           /\ bad' = (bad \/ \E q \in Ranks : inp[q] # c[r])
           /\ out' = IF Two THEN [q \in Ranks |-> [out[q] EXCEPT ![r] = c[r]]]
                     ELSE [out EXCEPT ![r] = [s \in Ranks |-> c[r]]]
           /\ ph' = [ph EXCEPT ![r] = 2]
           /\ UNCHANGED <<c, arr, dep, inp>>

Depart(r) == /\ c[r] < C /\ ph[r] = 2
             /\ dep' = [dep EXCEPT ![r] = c[r] + 1]
             /\ ph' = [ph EXCEPT ![r] = 3]
             /\ UNCHANGED <<c, arr, inp, out, bad>>

Leave(r) == /\ c[r] < C /\ ph[r] = 3
            /\ SkipDepart \/ \A q \in Ranks : dep[q] >= c[r] + 1
            /\ c' = [c EXCEPT ![r] = c[r] + 1] /\ ph' = [ph EXCEPT ![r] = 0]
            /\ UNCHANGED <<arr, dep, inp, out, bad>>

Done == \A r \in Ranks : c[r] = C

Next == \/ \E r \in Ranks : Produce(r) \/ Data(r) \/ Depart(r) \/ Leave(r)
        \/ (Done /\ UNCHANGED vars)

Spec == Init /\ [][Next]_vars

CallsInStep == ~bad
=============================================================================
